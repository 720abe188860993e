"""The C ABI driven from a plain C program, no Python or PyTorch on its side (GPU).

``tests/c_abi/step_from_c.c`` allocates its own device buffers, fills the
descriptor table, step rows and slots as ``include/luma_b200.h`` documents,
and calls ``luma_step`` for two steps (first and quantized) on an fp32 and a
bf16 tensor.  The same inputs stepped through ``luma_b200.LUMA`` must give the
same params, codes and slot contents bit for bit — the boundary a non-Python
host would bind is the same path the package uses.
"""

import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c_abi", "step_from_c.c")
N0, N1 = 70001, 4099
SEED = -4_611_686_018_427_387_905


def _pattern(n, salt):
    i = np.arange(n, dtype=np.uint32)
    with np.errstate(over="ignore"):
        x = i * np.uint32(2654435761) ^ np.uint32((salt * 0x9E3779B9) & 0xFFFFFFFF)
        x ^= x >> np.uint32(15)
        x *= np.uint32(0x2C1B3C6D)
        x ^= x >> np.uint32(12)
    return (x & np.uint32(0xFFFFFF)).astype(np.float32) / np.float32(8388608.0) - np.float32(1.0)


def _build(tmp_path):
    exe = str(tmp_path / "step_from_c")
    cc = shutil.which("gcc") or shutil.which("cc")
    lib = os.path.join(ROOT, "luma_b200", "_lib")
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    subprocess.run([cc, "-O2", "-std=c11", "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(cuda, "include"), SRC, "-o", exe, "-L", lib, "-lluma_b200",
                    "-L", os.path.join(cuda, "lib64"), "-lcudart", "-lm", f"-Wl,-rpath,{lib}",
                    f"-Wl,-rpath,{os.path.join(cuda, 'lib64')}"], check=True)
    return exe


def test_c_program_matches_package_bit_exact(tmp_path):
    from luma_b200 import LUMA
    from luma_b200 import _lib
    _lib.lib()  # built, ABI checked
    exe = _build(tmp_path)
    out = tmp_path / "out.bin"
    r = subprocess.run([exe, str(out), str(SEED)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr

    p0 = torch.from_numpy(np.float32(0.02) * _pattern(N0, 1)).cuda()
    p1 = torch.from_numpy(np.float32(0.02) * _pattern(N1, 2)).to(torch.bfloat16).cuda()
    for p in (p0, p1):
        p.grad_dtype = None
    opt = LUMA([p0, p1], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    opt._base_seed = SEED
    for t in (1, 2):
        p0.grad = torch.from_numpy(np.float32(1e-3) * _pattern(N0, 10 + t)).to(torch.bfloat16).cuda()
        p1.grad = torch.from_numpy(np.float32(1e-3) * _pattern(N1, 20 + t)).to(torch.bfloat16).cuda()
        opt.step()
    torch.cuda.synchronize()

    raw = out.read_bytes()
    pos = 0

    def take(nbytes):
        nonlocal pos
        b = raw[pos:pos + nbytes]
        pos += nbytes
        return b

    c_p0 = np.frombuffer(take(N0 * 4), dtype=np.uint32)
    c_p1 = np.frombuffer(take(N1 * 2), dtype=np.uint16)
    c_qm0 = np.frombuffer(take(N0 * 2), dtype=np.int16)
    c_qw0 = np.frombuffer(take(N0 * 2), dtype=np.int16)
    c_qm1 = np.frombuffer(take(N1 * 2), dtype=np.int16)
    c_qw1 = np.frombuffer(take(N1 * 2), dtype=np.int16)
    c_slots = np.frombuffer(take(2 * _lib.SLOT_DTYPE.itemsize), dtype=np.uint8)
    assert pos == len(raw)
    assert np.array_equal(c_p0, p0.cpu().view(torch.int32).numpy().view(np.uint32))
    assert np.array_equal(c_p1, p1.cpu().view(torch.int16).numpy().view(np.uint16))
    s0, s1 = opt.state[p0], opt.state[p1]
    assert np.array_equal(c_qm0, s0["Q_m"].cpu().numpy()) and np.array_equal(c_qw0, s0["Q_w"].cpu().numpy())
    assert np.array_equal(c_qm1, s1["Q_m"].cpu().numpy()) and np.array_equal(c_qw1, s1["Q_w"].cpu().numpy())
    eng = next(iter(opt._engines.values()))
    py_slots = eng.slots[:2 * _lib.SLOT_DTYPE.itemsize].cpu().numpy()
    assert np.array_equal(c_slots, py_slots)
