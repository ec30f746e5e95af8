"""CUDA layer vs the CPU oracle on reduced batches of benchmark configurations 2-4.

Samples are independent, so a sub-batch exercises the same arithmetic as the
full configuration.  Forward results are compared bit for bit at a fixed
iteration count through the public API (presolve, row scaling, forward and
post-processing).  The implicit gradient of configuration 2 comes from GMRES
runs that meet their tolerance in both implementations; its dot products are
parallel sums on the GPU, so it is compared with a relative tolerance.
"""

from dataclasses import replace

import numpy as np
import pytest
import torch

from helpers import OracleLayer
from purin_b200 import LinearSolverConfig, prepare_projection
from purin_b200.metric import _scaled_problem
from purin_b200.workloads import make_workload

pytestmark = pytest.mark.gpu

DEV = "cuda"
FIELDS = ("y", "multipliers_eq", "multipliers_ineq", "slacks", "status", "iterations", "finite",
          "gradient_eligible")


def _tdt(dtype):
    return torch.float64 if dtype == np.float64 else torch.float32


def _t(a, dtype):
    return torch.as_tensor(np.ascontiguousarray(a, dtype=dtype), device=DEV)


def _layer(problem, cfg, batch, dtype):
    return prepare_projection(problem, method="chambolle-pock", config=cfg, batch_size=batch,
                              dtype=_tdt(dtype), backend=DEV)


def _assert_forward(got, expected, residual_factor=1.0):
    for field in FIELDS:
        np.testing.assert_array_equal(getattr(got, field).cpu().numpy(), expected[field],
                                      err_msg=field)
    np.testing.assert_allclose(got.residual_inf_norm.cpu().numpy(),
                               expected["residual_inf_norm"] * residual_factor, rtol=1e-6, atol=0)


def test_config3_network_flow_fp32():
    """5000-node, 20000-edge flow with coupling rows and capacity bounds (fp32)."""
    batch = 2
    w = make_workload(3, batch)
    cfg = replace(w.config, max_iterations=200)
    oracle = OracleLayer(w.problem, cfg, np.float32)
    expected, _ = oracle.solve(w.candidates, w.theta)
    layer = _layer(w.problem, cfg, batch, np.float32)
    got = layer.solve(_t(w.candidates, np.float32), _t(w.theta, np.float32))
    _assert_forward(got, expected)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_config4_weighted_distance(dtype):
    """WeightedDistance (w ~ U(0.5, 2)), 16 nnz per row, accelerated steps."""
    batch = 3
    w = make_workload(4, batch)
    diagonal = tuple(float(v) for v in w.weights)
    cfg = replace(w.config, max_iterations=300, metric_diagonal=diagonal)
    layer = _layer(w.problem, cfg, batch, dtype)
    got = layer.solve(_t(w.candidates, dtype), _t(w.theta, dtype))
    # The weighted projection is the Euclidean one of sqrt(w) * candidate onto the
    # problem whose column j is scaled by 1/sqrt(w_j) (metric.py:15-84, 158-182).
    factor = max(1.0, float(np.sqrt(max(diagonal))))
    root = np.sqrt(np.asarray(diagonal, dtype=dtype))
    base_cfg = replace(cfg, metric_diagonal=None, tolerance=cfg.tolerance / factor)
    oracle = OracleLayer(_scaled_problem(w.problem, 1 / np.sqrt(np.asarray(diagonal))), base_cfg,
                         dtype)
    expected, _ = oracle.solve(np.asarray(w.candidates, dtype=dtype) * root, w.theta)
    expected = dict(expected, y=expected["y"] / root)
    _assert_forward(got, expected, residual_factor=factor)


@pytest.mark.parametrize("dtype,samples", [(np.float64, 2), (np.float32, 4)])
def test_config4_wide_tiles_equal_one_sample_tiles(monkeypatch, dtype, samples):
    """Config 4's structure (0.98 MB in fp64) takes the wide tiles once the batch fills
    one per SM: 2 (fp64) or 4 (fp32) samples on 768 threads, lines ordered for their
    16-byte gathers.  The whole public solve then equals the one-sample tiles' bit for bit
    (every tile shape gives the oracle's bits: test_forward_tile_widths_match_oracle)."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    batch = samples * sms
    w = make_workload(4, batch)
    cfg = replace(w.config, max_iterations=60,
                  metric_diagonal=tuple(float(v) for v in w.weights))
    layer = _layer(w.problem, cfg, batch, dtype)
    assert layer._plan.forward_shape(layer._cfg, batch) == (samples, 768, True)
    wide = layer.solve(_t(w.candidates, dtype), _t(w.theta, dtype))
    monkeypatch.setenv("PURIN_CP_SAMPLES_PER_TILE", "1")
    monkeypatch.setenv("PURIN_CP_TILE_THREADS", "256")
    assert layer._plan.forward_shape(layer._cfg, batch) == (1, 256, True)
    narrow = layer.solve(_t(w.candidates, dtype), _t(w.theta, dtype))
    for field in FIELDS + ("residual_inf_norm",):
        np.testing.assert_array_equal(getattr(wide, field).cpu().numpy(),
                                      getattr(narrow, field).cpu().numpy(), err_msg=field)


def test_config2_forward_and_candidate_gradient():
    """fp64, n = 2048, loss 0.5 ||y - t||^2 with samples that converge (CP tolerance 1e-3)."""
    batch = 2
    w = make_workload(2, batch)
    cfg = replace(w.config, tolerance=1e-3, linear_solver=LinearSolverConfig(tolerance=1e-4))
    oracle = OracleLayer(w.problem, cfg, np.float64)
    expected, saved = oracle.solve(w.candidates, w.theta)
    assert expected["gradient_eligible"].all()
    stats = {}
    cot = expected["y"] - w.targets
    want = oracle.proj.vjp(saved, cot, stats=stats)["target"]
    assert (stats["code"] == 0).all()

    layer = _layer(w.problem, cfg, batch, np.float64)
    x = _t(w.candidates, np.float64).requires_grad_(True)
    theta = _t(w.theta, np.float64)
    y = layer(x, theta)
    np.testing.assert_array_equal(y.detach().cpu().numpy(), expected["y"])
    (0.5 * ((y - _t(w.targets, np.float64)) ** 2).sum()).backward()
    got = x.grad.cpu().numpy()
    status, _ = layer._last_linear
    assert (status.cpu().numpy() == 0).all()
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= 1e-6, err
