"""CPU-only checks of the host side: the C-ABI library loads, exports every
symbol include/bsa.h declares, validates arguments without a GPU, and the
Python layer refuses CPU tensors instead of falling back."""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT


def _declared():
    h = open(os.path.join(ROOT, "include", "bsa.h")).read()
    return sorted(set(re.findall(r"^\s*(?:bsa_status|size_t|int32_t|const char \*)\s*\*?\s*(bsa_\w+)\(",
                                 h, re.M)))


def test_header_symbols_exported():
    import _bsa
    L = _bsa.lib()
    names = _declared()
    assert len(names) >= 12, names
    for n in names:
        assert hasattr(L, n), n
    assert set(names) <= set(_bsa.SYMBOLS), set(names) - set(_bsa.SYMBOLS)
    assert L.bsa_version() >= 100


def test_struct_layouts_match_the_header(tmp_path):
    """The ctypes mirrors in _bsa must have the sizes and field offsets that a C
    compiler gives the structs of include/bsa.h."""
    import subprocess
    import _bsa
    structs = {"bsa_view": _bsa.View, "bsa_attn_args": _bsa.AttnArgs, "bsa_pool_args": _bsa.PoolArgs,
               "bsa_select_args": _bsa.SelectArgs, "bsa_lsh_args": _bsa.LshArgs,
               "bsa_csr_args": _bsa.CsrArgs, "bsa_rope_args": _bsa.RopeArgs,
               "bsa_decode_args": _bsa.DecodeArgs, "bsa_scores_args": _bsa.ScoresArgs,
               "bsa_qmax_args": _bsa.QmaxArgs, "bsa_centroid_args": _bsa.CentroidArgs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "bsa.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append('printf("%s %%zu\\n", sizeof(%s));' % (cname, cname))
        for f, _ in cls._fields_:
            lines.append('printf("%s.%s %%zu\\n", offsetof(%s, %s));' % (cname, f, cname, f))
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                  check=True).stdout.splitlines())
    for cname, cls in structs.items():
        assert int(got[cname]) == ctypes.sizeof(cls), cname
        for f, _ in cls._fields_:
            assert int(got[cname + "." + f]) == getattr(cls, f).offset, (cname, f)


def test_validation_errors_without_gpu():
    import _bsa
    L = _bsa.lib()
    a = _bsa.AttnArgs()
    a.dtype = 7
    assert L.bsa_attn_fwd(ctypes.byref(a), None) == _bsa.ERR_DTYPE
    assert b"dtype" in L.bsa_last_error()
    a.dtype = _bsa.BF16
    a.B = a.Hq = a.Hkv = 1
    a.L, a.D, a.bs, a.nblk, a.kk = 100, 64, 64, 3, 2      # nblk != ceil(L/bs)
    a.scale = 0.125
    assert L.bsa_attn_fwd(ctypes.byref(a), None) == _bsa.ERR_SHAPE
    a.nblk, a.Hq, a.Hkv = 2, 3, 2                          # Hq % Hkv != 0
    assert L.bsa_attn_fwd(ctypes.byref(a), None) == _bsa.ERR_SHAPE
    s = _bsa.SelectArgs()
    s.layout, s.nblk, s.topk, s.sink = _bsa.SEL_FINISH, 10, 32, 1
    assert L.bsa_select_width(ctypes.byref(s)) == 12
    s.layout = _bsa.SEL_SSA
    assert L.bsa_select_width(ctypes.byref(s)) == 10
    s.topk = 33
    assert L.bsa_select(ctypes.byref(s), None) in (_bsa.ERR_ARG, _bsa.ERR_UNSUPPORTED, _bsa.ERR_SHAPE)
    assert L.bsa_status_decode(_bsa.DEVERR_INDEX) == _bsa.ERR_INDEX
    assert L.bsa_status_decode(_bsa.DEVERR_TIMEOUT | _bsa.DEVERR_INDEX) == _bsa.ERR_TIMEOUT


def test_no_cpu_fallback():
    import triton_kernel as tk
    q = torch.randn(1, 1, 128, 64)
    sel = torch.zeros(1, 2, 1, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        tk.bsattn_forward(q, q, q, sel)
