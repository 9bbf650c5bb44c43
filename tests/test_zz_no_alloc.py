"""The allocation-free CSR transpose (bsa_sel_csr_noalloc) against the regular
entry point (bsa_sel_csr with a caller workspace).

bsa_sel_csr_noalloc exists for callers that may not allocate device memory
where they build the transpose (a locked or exhausted pool, a host runtime
that owns all device allocations); it keeps its scratch in a fixed device
array inside the library.  The check: two calls in a row, each through the C
ABI, must give the same row_ptr / col as the regular entry point (integer
output, so the tolerance is exact equality), the second call with a smaller
selection so that leftovers of the first call in the shared array would show.
Oversized selections must be rejected before any launch.

This file is named to be collected last."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _args(sel, bs, causal, mode):
    import _bsa
    c = _bsa.CsrArgs()
    c.B, c.Hs, c.nblk, c.kk = sel.shape
    c.sel_sb, c.sel_sh, c.sel_sn = sel.stride(0), sel.stride(1), sel.stride(2)
    c.bs, c.L, c.mask_mode, c.causal = bs, c.nblk * bs, mode, 1 if causal else 0
    c.sel = sel.data_ptr()
    nb = c.B * c.Hs * c.nblk
    row_ptr = torch.full((nb + 1,), -7, dtype=torch.int32, device=sel.device)
    col = torch.full((nb * c.kk,), -7, dtype=torch.int32, device=sel.device)
    c.row_ptr, c.col = row_ptr.data_ptr(), col.data_ptr()
    return c, row_ptr, col


def _regular(sel, bs, causal, mode):
    import _bsa
    c, rp, col = _args(sel, bs, causal, mode)
    L = _bsa.lib()
    n = L.bsa_csr_workspace(ctypes.byref(c))
    ws = torch.empty(n, dtype=torch.uint8, device=sel.device)
    st = L.bsa_sel_csr(ctypes.byref(c), ctypes.c_void_p(ws.data_ptr()), n, _bsa._stream())
    assert st == _bsa.OK, L.bsa_last_error()
    return rp, col


def _noalloc(sel, bs, causal, mode):
    import _bsa
    c, rp, col = _args(sel, bs, causal, mode)
    L = _bsa.lib()
    st = L.bsa_sel_csr_noalloc(ctypes.byref(c), _bsa._stream())
    assert st == _bsa.OK, L.bsa_last_error()
    return rp, col


def _sel(seed, B, H, nblk, kk, dev):
    g = torch.Generator().manual_seed(seed)
    s = torch.randint(0, nblk, (B, H, nblk, kk), generator=g, dtype=torch.int32)
    s[..., 0] = torch.arange(nblk, dtype=torch.int32)
    return s.to(dev)


@pytest.mark.parametrize("mode,causal", [(0, True), (1, True)])
def test_noalloc_matches_regular_twice(cuda, mode, causal):
    for seed, shape in ((1, (2, 4, 600, 17)), (2, (1, 2, 130, 9))):
        sel = _sel(seed, *shape, cuda)
        rp_ref, col_ref = _regular(sel, 64, causal, mode)
        rp, col = _noalloc(sel, 64, causal, mode)
        torch.cuda.synchronize()
        n = int(rp_ref[-1].item())
        assert torch.equal(rp, rp_ref)
        assert torch.equal(col[:n], col_ref[:n])


def test_noalloc_rejects_oversized_selection(cuda):
    import _bsa
    sel = torch.zeros(1, 1, 1 << 16, 64, dtype=torch.int32, device=cuda)  # 4 M entries
    c, rp, col = _args(sel, 64, True, 0)
    L = _bsa.lib()
    st = L.bsa_sel_csr_noalloc(ctypes.byref(c), _bsa._stream())
    assert st == _bsa.ERR_UNSUPPORTED
    assert b"scratch" in L.bsa_last_error()
    torch.cuda.synchronize()
    assert int(rp[0].item()) == -7          # nothing was launched
