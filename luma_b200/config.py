"""Constants and launch configuration of the CUDA backend.

The grid constants are the reference's (src/luma_optimizer/config.py:23-25).
``get_kernel_config`` keeps the reference's function name (config.py:35-73)
but describes this backend's launch shape: 256-thread CTAs, one octet (8
elements, 128-bit loads) per thread per iteration, a persistent grid of
``SMs x resident CTAs`` per pass.
"""

from __future__ import annotations

from .hostmath import K_M, K_W, SCALE_FLOOR_M  # noqa: F401

THREADS_PER_CTA = 256
ELEMS_PER_THREAD = 8


def get_kernel_config(device=None) -> dict[str, int]:
    """Launch parameters of the two step kernels on ``device``."""
    cfg = {"BLOCK_SIZE": THREADS_PER_CTA * ELEMS_PER_THREAD,
           "threads_per_cta": THREADS_PER_CTA,
           "elems_per_thread": ELEMS_PER_THREAD}
    try:
        import torch
        if device is not None and torch.device(device).type == "cuda" and torch.cuda.is_available():
            cfg["sms"] = torch.cuda.get_device_properties(device).multi_processor_count
    except Exception:  # noqa: BLE001 - informational only
        pass
    return cfg
