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


@pytest.mark.parametrize("gdt", [torch.float32, torch.bfloat16, torch.float16])
def test_clip_coef_is_the_multiplier_clip_grad_norm_applies(gdt):
    """clip_grad_norm_ stores round_to_dtype(fl32(g) * coef) with the coef
    clip_grad_coef returns (the rounding model the fused kernels follow)."""
    from luma_b200 import clip_grad_coef
    gen = torch.Generator().manual_seed(3)
    ps = [torch.nn.Parameter(torch.zeros(n)) for n in (1000, 77, 5)]
    for p in ps:
        p.grad_dtype = None
        p.grad = (torch.randn(p.shape, generator=gen) * 0.5).to(gdt)
    grads = [p.grad.clone() for p in ps]
    norm, coef = clip_grad_coef(ps, 0.1)
    assert all(torch.equal(p.grad, g) for p, g in zip(ps, grads))
    ref_norm = torch.nn.utils.clip_grad_norm_(ps, 0.1)
    assert torch.equal(norm, ref_norm)
    assert coef.dtype == gdt and float(coef) < 1.0  # the norm's dtype follows the grads'
    for p, g in zip(ps, grads):
        assert torch.equal(p.grad, (g.float() * coef.float()).to(gdt))
