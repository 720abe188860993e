"""luma_b200 — LUMA (Log-space Unbiased Momentum AdamW) optimizer step for B200.

Drop-in for ``luma_optimizer`` (IgorYashch/LUMA): ``LUMA`` keeps the
reference's constructor, state layout and checkpoint format; its step runs as
two hand-written sm_100a kernels over all parameters (``libluma_b200.so``).
"""

from .config import K_M, K_W, SCALE_FLOOR_M, get_kernel_config
from .optimizer import LUMA
from . import torch_op  # registers torch.ops.luma_b200.step
from .clip import clip_grad_coef
from . import amp  # scaler_step: GradScaler.unscale_ fused into the step

__all__ = ["LUMA", "amp", "clip_grad_coef", "get_kernel_config", "K_M", "K_W", "SCALE_FLOOR_M"]
__version__ = "0.1.0"
