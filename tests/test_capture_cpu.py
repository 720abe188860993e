"""Host side of capturable mode and the custom op (CPU): the vectorised row
table equals the per-step rows byte for byte, the op is registered with its
schema, and the constructor validates its options."""

import numpy as np
import pytest
import torch

from luma_b200.hostmath import rows_array, step_row, step_rows


@pytest.mark.parametrize("hp", [(1e-3, 0.9, 0.999, 1e-8, 0.01), (3e-4, 0.95, 0.98, 1e-6, 0.1),
                                (1.0, 0.0, 0.5, 1.0, 0.0), (0.0, 0.9, 0.999, 1e-8, 0.0)])
def test_row_table_equals_per_step_rows(hp):
    steps = np.concatenate([np.arange(1, 5001), np.array([65535, 65536, 131071, 131072])])
    table = step_rows(steps, *hp)
    ref = rows_array([step_row(int(t), *hp) for t in steps])
    assert np.array_equal(table.view(np.uint8), ref.view(np.uint8))


def test_custom_op_registered():
    import luma_b200  # noqa: F401
    schema = str(torch.ops.luma_b200.step.default._schema)
    for arg in ("Tensor(a0!)[] params", "Tensor(a2!)[] q_m", "Tensor(a3!)[] q_w",
                "Tensor(a4!) slots", "Tensor(a5!) counters", "Tensor row_table"):
        assert arg in schema


def test_capturable_options_validated():
    from luma_b200 import LUMA
    p = [torch.nn.Parameter(torch.zeros(4))]
    with pytest.raises(ValueError, match="capture_steps"):
        LUMA(p, capturable=True, capture_steps=0)
    opt = LUMA(p, capturable=True, capture_steps=16)
    assert opt.capturable and opt.capture_steps == 16
    with pytest.raises(RuntimeError, match="capturable=True"):
        LUMA(p).step_op_args()
