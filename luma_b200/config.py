"""Constants and launch configuration of the CUDA backend.

The grid constants are the reference's (src/luma_optimizer/config.py:23-25).
``get_kernel_config`` keeps the reference's function name and its three keys
(config.py:35-73: ``BLOCK_SIZE``, ``num_warps``, ``num_stages``) but reports
this backend's launch shape, read from the compiled library so it cannot
drift from the kernels:

* ``BLOCK_SIZE`` — elements one pass-2 CTA steps per loop iteration (its
  threads x two Philox pairs of 2 elements each);
* ``num_warps`` — warps per pass-2 CTA;
* ``num_stages`` — pass-2 shared-memory staging depth (iterations of
  ``cp.async`` copies in flight);

plus the per-pass details (pass 1 runs 1024-thread CTAs over octets of 8
elements, 2 staging stages), one persistent CTA per SM for both passes, and
``sms`` when a CUDA device is given.
"""

from __future__ import annotations

from . import _lib
from .hostmath import K_M, K_W, SCALE_FLOOR_M  # noqa: F401


def get_kernel_config(device=None) -> dict[str, int]:
    """Launch parameters of the two step kernels (and ``sms`` of ``device``)."""
    lc = _lib.launch_config()
    cfg = {"BLOCK_SIZE": lc["pass2_threads"] * lc["pass2_elems_per_thread"],
           "num_warps": lc["pass2_threads"] // 32,
           "num_stages": lc["pass2_stages"]}
    cfg.update(lc)
    try:
        import torch
        if device is not None and torch.device(device).type == "cuda" and torch.cuda.is_available():
            cfg["sms"] = torch.cuda.get_device_properties(device).multi_processor_count
    except Exception:  # noqa: BLE001 - informational only
        pass
    return cfg
