"""Committed golden fixtures (tests/golden/): the oracle on CPU, the CUDA layer on GPU."""

import json
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest

from helpers import OracleLayer, make_problem
from purin_b200 import ChambollePockConfig
from purin_b200.workloads import make_workload

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURES = [("oracle_config0.npz", 0, 4, np.float64, 500),
            ("oracle_config1_f32.npz", 1, 2, np.float32, 100)]


@pytest.mark.parametrize("name,index,batch,dtype,iters", FIXTURES, ids=[f[0] for f in FIXTURES])
def test_oracle_reproduces_fixture(name, index, batch, dtype, iters):
    w = make_workload(index, batch)
    result, _ = OracleLayer(w.problem, replace(w.config, max_iterations=iters), dtype).solve(
        w.candidates, w.theta)
    fixture = np.load(GOLDEN / name)
    for key in fixture.files:
        np.testing.assert_array_equal(result[key], fixture[key], err_msg=key)


def test_reference_cases_on_the_oracle():
    cases = json.loads((GOLDEN / "reference_cases.json").read_text())
    case = cases["affine_projection"]
    layer = OracleLayer(make_problem(), ChambollePockConfig(tolerance=1e-9, max_iterations=3000))
    target, theta = np.array(case["target"]), np.array(case["parameters"])
    np.testing.assert_allclose(layer(target, theta), case["y"], atol=case["atol_y"], rtol=0)
    np.testing.assert_allclose(layer.target_jacobian(target, theta)[0], case["jacobian"],
                               atol=case["atol_jacobian"], rtol=0)


@pytest.mark.gpu
@pytest.mark.parametrize("name,index,batch,dtype,iters", FIXTURES, ids=[f[0] for f in FIXTURES])
def test_cuda_layer_reproduces_fixture(name, index, batch, dtype, iters):
    import torch

    from purin_b200 import prepare_projection

    w = make_workload(index, batch)
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    layer = prepare_projection(w.problem, method="chambolle-pock",
                               config=replace(w.config, max_iterations=iters), batch_size=batch,
                               dtype=tdt, backend="cuda")
    got = layer.solve(torch.as_tensor(w.candidates, dtype=tdt, device="cuda"),
                      torch.as_tensor(w.theta, dtype=tdt, device="cuda"))
    fixture = np.load(GOLDEN / name)
    for key in fixture.files:
        np.testing.assert_array_equal(getattr(got, key).cpu().numpy(), fixture[key], err_msg=key)
