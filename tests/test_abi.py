"""The C-ABI boundary without a GPU: the library loads, exports every symbol
include/qtts_b200.h declares, its ctypes structs have the C layout, and bad
arguments come back as status codes (no CUDA call is reached)."""

import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

from test_stateful_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qtts_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^int (qtts_[a-z0-9_]+)\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert declared == sorted(_lib.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (qtts_[a-z0-9_]+)$", out, flags=re.M)))
    assert exported == declared


def test_struct_layouts_match_c():
    """Compile a probe against the header with gcc and compare sizeof/offsetof."""
    probe = r"""
#include <stdio.h>
#include <stddef.h>
#include "qtts_b200.h"
int main(void) {
  printf("%zu %zu %zu %zu\n", sizeof(qtts_paged_state), sizeof(qtts_qkv_epilogue), sizeof(qtts_model_desc),
         sizeof(qtts_step_io));
  printf("%zu %zu %zu %zu\n", offsetof(qtts_model_desc, pool), offsetof(qtts_model_desc, max_prefill_rows),
         offsetof(qtts_step_io, noise_seed), offsetof(qtts_step_io, launches));
  printf("%zu %zu %zu %zu %zu\n", sizeof(qtts_c2w_desc), offsetof(qtts_c2w_desc, rvq_tables),
         offsetof(qtts_c2w_desc, up_w), offsetof(qtts_c2w_desc, res_b2), offsetof(qtts_c2w_desc, final_b));
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(src, "w").write(probe)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    sizes = [int(v) for v in lines[0].split()]
    offs = [int(v) for v in lines[1].split()]
    assert sizes == [C.sizeof(_lib.PagedState), C.sizeof(_lib.QkvEpilogue), C.sizeof(_lib.ModelDesc),
                     C.sizeof(_lib.StepIO)]
    assert offs == [_lib.ModelDesc.pool.offset, _lib.ModelDesc.max_prefill_rows.offset,
                    _lib.StepIO.noise_seed.offset, _lib.StepIO.launches.offset]
    c2w = [int(v) for v in lines[2].split()]
    D = _lib.C2wDesc
    assert c2w == [C.sizeof(D), D.rvq_tables.offset, D.up_w.offset, D.res_b2.offset, D.final_b.offset]


def test_invalid_arguments_return_status_codes():
    lib = _lib.load()
    assert lib.qtts_version() >= 1
    rc = lib.qtts_gemm(None, None, 64, 2048, None, 2048, _lib.EPI_F32, None, None, None, None, None)
    assert rc == _lib.ERR_INVALID
    assert "gemm" in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.check(rc, "gemm")
    st = _lib.PagedState()
    assert lib.qtts_sched_init(C.byref(st), None) == _lib.ERR_INVALID
    assert lib.qtts_engine_create(None, None) == _lib.ERR_INVALID
    assert lib.qtts_engine_step(None, None, None) == _lib.ERR_INVALID
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_POOL_EXHAUSTED, "append")


def test_no_cpu_fallback():
    """Without a CUDA device the product path refuses to run rather than computing on the host:
    the executor will not construct, and the kernel wrappers reject host tensors before any call."""
    import torch

    from test_stateful_b200 import ops
    from test_stateful_b200.runtime.executor import B200Executor

    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="no CPU path"):
            B200Executor(max_batch_size=1, max_seq_len=16)
    x = torch.zeros(64, 2048, dtype=torch.bfloat16)
    w = torch.zeros(2048, 2048, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        ops.gemm(x, w)
