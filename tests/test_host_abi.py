"""Host-side logic and the C ABI boundary — CPU (no GPU calls).

* the shared library loads and exports every function include/luma_b200.h
  declares; the ABI version and struct sizes agree with the Python mirrors;
* every struct field offset in the header (compiled with gcc, offsetof)
  equals the numpy mirror's offset;
* host scalar math (grid precompute, per-step rows) reproduces the float32
  roundings the reference's tensor ops apply to Python scalars;
* descriptor-table construction (octet prefix sums, 128-bit alignment flag).
"""

import ctypes
import math
import os
import re
import subprocess

import numpy as np
import pytest
import torch

from luma_b200 import _lib
from luma_b200.engine import Segment, build_desc_table
from luma_b200.hostmath import grid_record, precompute, step_row

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "luma_b200.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(luma_\w+)\s*\(", src, re.M)))


def test_library_exports_every_declared_symbol():
    h = _lib.lib()
    names = declared_functions()
    assert set(_lib.EXPORTED) <= set(names)
    for n in names:
        assert hasattr(h, n), f"{n} declared in luma_b200.h but not exported"


def test_abi_version_and_struct_sizes():
    h = _lib.lib()
    assert h.luma_abi_version() == _lib.ABI_VERSION
    out = (ctypes.c_int64 * 5)()
    assert h.luma_struct_sizes(out, 5) == 5
    assert tuple(out) == _lib.EXPECTED_SIZES
    assert h.luma_last_error() == b""


def test_invalid_arguments_rejected_without_gpu():
    h = _lib.lib()
    assert h.luma_step(None, None) == _lib.LUMA_ERR_INVALID
    assert b"NULL" in h.luma_last_error()
    a = _lib.LumaStepArgs()
    a.n_desc = -1
    assert h.luma_step(ctypes.byref(a), None) == _lib.LUMA_ERR_INVALID
    a.n_desc = 0  # nothing to do: OK without touching the device
    assert h.luma_step(ctypes.byref(a), None) == _lib.LUMA_OK
    a.n_desc, a.total_octets, a.n_rows = 3, 10, 1
    assert h.luma_step(ctypes.byref(a), None) == _lib.LUMA_ERR_INVALID  # NULL tables
    assert h.luma_decode(None, None, -1, 0, 0, 0, 0, None, None, None) == _lib.LUMA_ERR_INVALID


def _c_offsets(struct, fields, tmp_path):
    src = tmp_path / "off.c"
    body = "\n".join(f'  printf("%zu\\n", offsetof({struct}, {f}));' for f in fields)
    src.write_text(f'#include <stddef.h>\n#include <stdio.h>\n#include "luma_b200.h"\n'
                   f'int main(void) {{\n  printf("%zu\\n", sizeof({struct}));\n{body}\n  return 0;\n}}\n')
    exe = tmp_path / "off"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True,
                                           text=True).stdout.split()]
    return vals[0], vals[1:]


@pytest.mark.parametrize("struct,dtype", [("LumaTensorDesc", _lib.DESC_DTYPE),
                                          ("LumaStepRow", _lib.ROW_DTYPE),
                                          ("LumaGrid", _lib.GRID_DTYPE),
                                          ("LumaSlot", _lib.SLOT_DTYPE)])
def test_header_layout_matches_python_mirror(struct, dtype, tmp_path):
    fields = list(dtype.names)
    size, offs = _c_offsets(struct, fields, tmp_path)
    assert size == dtype.itemsize
    assert offs == [dtype.fields[f][1] for f in fields]


def test_step_args_layout(tmp_path):
    fields = [f for f, _ in _lib.LumaStepArgs._fields_]
    size, offs = _c_offsets("LumaStepArgs", fields, tmp_path)
    assert size == ctypes.sizeof(_lib.LumaStepArgs)
    assert offs == [getattr(_lib.LumaStepArgs, f).offset for f in fields]


def test_step_row_scalars():
    f = np.float32
    r = step_row(1, 1e-3, 0.9, 0.999, 1e-8, 0.01)
    assert r[0] == 1 and r[1] == 1e-8
    assert r[2] == f(0.9) and r[3] == f(1.0 - 0.9) and r[4] == f(0.999) and r[5] == f(1.0 - 0.999)
    assert r[6] == f(1.0 - 0.01 * 1e-3)
    assert r[7] == f(-(1e-3 / (1.0 - 0.9)))
    assert r[8] == f(1.0 / (1.0 - 0.999))
    assert r[9] == f(1e-8) and r[10] == f(1e8)
    r7 = step_row(7, 3e-4, 0.9, 0.95, 1e-6, 0.1)
    assert r7[7] == f(-(3e-4 / (1.0 - 0.9 ** 7)))
    assert r7[8] == f(1.0 / (1.0 - 0.95 ** 7))
    r0 = step_row(3, 0.0, 0.9, 0.999, 1e-8, 0.0)
    assert r0[6] == f(1.0) and r0[7] == 0.0 and math.copysign(1.0, r0[7]) == -1.0


@pytest.mark.parametrize("S_m,S_v,eps", [(1e-9, 0.0, 1e-8), (0.5, 1e-6, 1e-8), (3.0, 2.5, 1e-8),
                                         (1e4, 1e8, 1e-10), (1e-3, 1e-40, 1.0)])
def test_grid_record(S_m, S_v, eps):
    f = np.float32
    g = grid_record(S_m, S_v, eps)
    w_min, dm, z_m, dw, z_w = precompute(S_m, S_v, eps)
    assert g["S_m"] == S_m and g["S_v"] == S_v and g["eps"] == eps
    assert g["dm"] == f(dm) and g["inv_dm"] == f(1 / dm) and g["inv_zm"] == f(1 / z_m)
    assert g["s_m32"] == f(S_m) and g["w_min"] == f(w_min) and g["inv_wmin"] == f(1 / w_min)
    assert g["dw_pos"] == (dw > 0)
    if dw > 0:
        assert g["dw"] == f(dw) and g["inv_dw"] == f(1 / dw) and g["inv_zw"] == f(1 / z_w)
    else:
        assert g["dw"] == 0 and g["inv_zw"] == 1


def test_desc_table_octets_and_alignment():
    buf = torch.zeros(4096)
    q = torch.zeros(8192, dtype=torch.int16)
    segs = []
    for k, (off, n) in enumerate([(0, 17), (64, 8), (129, 100), (512, 1)]):
        segs.append(Segment(buf[off:off + n], buf[off:off + n], q[off:off + n], q[off:off + n],
                            param_id=k, row=0, slot=k))
    table, total = build_desc_table(segs)
    assert list(table["numel"]) == [17, 8, 100, 1]
    assert list(table["oct_begin"]) == [0, 3, 4, 17]
    assert total == 18
    assert list(table["vec_ok"]) == [1, 1, 0, 1]  # element offset 129 breaks 16-byte alignment
    assert list(table["param_dtype"]) == [0] * 4 and list(table["slot"]) == [0, 1, 2, 3]


def test_column_table_equals_segment_table():
    """The optimizer's per-step fast path (descriptor columns) builds the same
    bytes as the Segment path for the same tensors, dtypes, rows and slots."""
    from luma_b200.engine import Columns, build_desc_table_columns, dtype_code
    rng = np.random.default_rng(4)
    buf = torch.zeros(1 << 16)
    hb = torch.zeros(1 << 16, dtype=torch.bfloat16)
    q = torch.zeros(1 << 17, dtype=torch.int16)
    segs, cols = [], Columns()
    off = 0
    for k in range(40):
        n = int(rng.integers(1, 600))
        p = (buf if k % 2 else hb)[off:off + n]
        g = (hb if k % 3 else buf)[off + 1:off + 1 + n] if k % 5 == 0 else (hb if k % 3 else buf)[off:off + n]
        m, w = q[2 * off:2 * off + n], q[2 * off + n:2 * off + 2 * n]
        row, slot = int(rng.integers(0, 3)), 39 - k
        segs.append(Segment(p, g, m, w, param_id=k, row=row, slot=slot))
        cols.statics.append((p.data_ptr(), m.data_ptr(), w.data_ptr(), n, k, slot,
                             dtype_code(p.dtype)))
        cols.grad_ptrs.append(g.data_ptr())
        cols.grad_codes.append(dtype_code(g.dtype))
        cols.rows.append(row)
        off += n + int(rng.integers(0, 9))
    t1, n1 = build_desc_table(segs)
    t2, n2 = build_desc_table_columns(cols)
    assert n1 == n2 and t1.tobytes() == t2.tobytes()


def test_new_entry_points_reject_bad_arguments_without_gpu():
    h = _lib.lib()
    assert h.luma_error_flags(None, 0) == _lib.LUMA_ERR_INVALID
    assert h.luma_arith_selfcheck(16, 0, None, None) == _lib.LUMA_ERR_INVALID
    assert h.luma_ipc_export(None, None, None) == _lib.LUMA_ERR_INVALID
    assert h.luma_ipc_open(None, None) == _lib.LUMA_ERR_INVALID
    assert h.luma_ipc_close(None) == _lib.LUMA_ERR_INVALID
    assert h.luma_copy_async(None, None, 0, None) == _lib.LUMA_OK  # nothing to copy
    assert h.luma_copy_async(None, None, 16, None) == _lib.LUMA_ERR_INVALID
    assert b"NULL" in h.luma_last_error()


def test_step_args_carry_capturable_scale_and_found_inf_fields():
    a = _lib.LumaStepArgs()
    names = [f for f, _ in _lib.LumaStepArgs._fields_]
    assert names[-3:] == ["step_counters", "grad_scale", "found_inf"]
    assert a.step_counters is None and a.grad_scale is None and a.found_inf is None
    assert ctypes.sizeof(a) == 104


def test_launch_config_matches_kernel_constants():
    from luma_b200 import get_kernel_config
    lc = _lib.launch_config()
    assert set(lc) == set(_lib.LAUNCH_KEYS)
    assert lc["ctas_per_sm"] == 1 and lc["pass1_elems_per_thread"] == 8
    assert lc["pass2_elems_per_thread"] == 4
    assert lc["pass1_threads"] % 32 == 0 and lc["pass2_threads"] % 32 == 0
    cfg = get_kernel_config()
    assert cfg["BLOCK_SIZE"] == lc["pass2_threads"] * 4
    assert cfg["num_warps"] == lc["pass2_threads"] // 32
    assert cfg["num_stages"] == lc["pass2_stages"]
    src = open(os.path.join(ROOT, "luma_b200", "csrc", "luma_step.cu")).read()
    m1 = re.search(r"constexpr int kThreadsPass1 = (\d+);", src)
    m2 = re.search(r"constexpr int kThreadsPass2 = (\d+);", src)
    assert int(m1.group(1)) == lc["pass1_threads"] and int(m2.group(1)) == lc["pass2_threads"]


def test_plain_c_consumer_builds_against_the_header(tmp_path):
    """``tests/c_abi/step_from_c.c`` (the C host the GPU test runs) compiles as
    warning-free C11 against ``include/luma_b200.h`` and links the library."""
    lib = os.path.join(ROOT, "luma_b200", "_lib")
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(cuda, "include"), os.path.join(ROOT, "tests", "c_abi", "step_from_c.c"),
                    "-o", str(tmp_path / "step_from_c"), "-L", lib, "-lluma_b200",
                    "-L", os.path.join(cuda, "lib64"), "-lcudart", "-lm", f"-Wl,-rpath,{lib}"], check=True)
