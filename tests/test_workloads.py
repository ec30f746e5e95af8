"""Synthetic workloads: a sample's data depends on its global index only.

A multi-GPU run gives rank r the samples [r B, (r + 1) B) of one global batch;
each rank generates only its slice, which must equal the same rows of the
whole batch generated at once.
"""

import numpy as np
import pytest

from purin_b200.workloads import SAMPLE_BLOCK, dense_workload, make_workload, qp_workload


@pytest.mark.parametrize("index", [0, 2, 3])
def test_slices_equal_rows_of_the_whole_batch(index):
    whole = make_workload(index, 3 * SAMPLE_BLOCK // 2 + 5)
    for offset, batch in ((0, 1), (7, SAMPLE_BLOCK), (SAMPLE_BLOCK - 1, 2), (SAMPLE_BLOCK + 3, 9)):
        part = make_workload(index, batch, offset=offset)
        rows = slice(offset, offset + batch)
        for name in ("theta", "candidates", "targets"):
            np.testing.assert_array_equal(getattr(part, name), getattr(whole, name)[rows],
                                          err_msg=f"{name} at offset {offset}")
        assert part.problem.name == whole.problem.name


def test_structure_is_shared_by_every_slice():
    a = make_workload(4, 2)
    b = make_workload(4, 2, offset=1000)
    np.testing.assert_array_equal(a.weights, b.weights)
    assert (a.problem.A_ineq != b.problem.A_ineq).nnz == 0
    assert not np.array_equal(a.candidates, b.candidates)


def test_float32_arrays_are_the_rounded_float64_ones():
    a = make_workload(4, 3, offset=5)
    b = make_workload(4, 3, offset=5, array_dtype=np.float32)
    np.testing.assert_array_equal(a.candidates.astype(np.float32), b.candidates)


def test_qp_and_dense_slices():
    q_all, q_part = qp_workload(70), qp_workload(6, offset=64)
    for k in (1, 2, 4, 7):
        np.testing.assert_array_equal(q_all[k][64:], q_part[k])
    d_all, d_part = dense_workload(70), dense_workload(6, offset=64)
    for x, y in zip(d_all, d_part):
        np.testing.assert_array_equal(x[64:], y)
