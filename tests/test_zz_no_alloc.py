"""bfp200_matvec_noalloc -- the matvec for callers that cannot allocate
device memory (their own allocator or memory pool owns every byte, or they
cannot take cudaMalloc's implicit synchronisation).  It must return exactly
what the allocating entry point bfp200_matvec returns, call after call, with
its scratch kept in the library's fixed device array, and what the oracle's
restatement of matvec_hw_golden (gen_smollm_blockfp_full.py:217-233)
returns.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

import inputs
from oracle import bfp_oracle as O

pytestmark = pytest.mark.gpu


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_noalloc_matches_allocating_entry_point():
    import torch
    from bfp200 import _lib, ops
    L = _lib.lib()
    for D_out, D_in, B in [(576, 576, 1), (1536, 576, 8), (576, 1536, 3), (192, 576, 64)]:
        W_m, W_e = inputs.sweep_weights(D_out, D_in)
        X_m, X_e = inputs.sweep_x(D_in, B, D_out)
        want_m, want_e = ops.matvec(X_m, X_e, W_m, W_e)          # existing entry point (bit-exact path)
        dWm, dWe, dXm, dXe = (_dev(torch, a) for a in (W_m, W_e, X_m, X_e))
        for call in range(2):                                     # two calls in a row share the scratch
            om = torch.full((B, D_out), 7, dtype=torch.int16, device="cuda")
            oe = torch.full((B, D_out // 16), 7, dtype=torch.int8, device="cuda")
            torch.cuda.synchronize()
            rc = L.bfp200_matvec_noalloc(dXm.data_ptr(), dXe.data_ptr(), dWm.data_ptr(), dWe.data_ptr(),
                                         D_out, D_in, B, om.data_ptr(), oe.data_ptr(), None)
            assert rc == 0, _lib.last_error()
            torch.cuda.synchronize()
            assert np.array_equal(om.cpu().numpy(), want_m), (D_out, D_in, B, call)
            assert np.array_equal(oe.cpu().numpy(), want_e), (D_out, D_in, B, call)
        # every column against the oracle
        got = O.tile_decode(om.cpu().numpy().reshape(-1), oe.cpu().numpy().reshape(-1)).reshape(B, D_out)
        assert np.array_equal(got, O.matvec_cols(X_m, X_e, W_m, W_e)), (D_out, D_in, B)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch
    from bfp200 import _lib
    L = _lib.lib()
    x = torch.zeros(16, dtype=torch.int16, device="cuda")
    rc = L.bfp200_matvec_noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 4096, 16, 65, x.data_ptr(),
                                 x.data_ptr(), None)
    assert rc == _lib.EINVAL and "exceeds" in _lib.last_error()


def test_noalloc_rejects_misaligned_pointers():
    # a pointer carved out of a caller's pool at a 2-byte offset is refused on
    # the host (no kernel runs), so the CUDA context stays usable
    import torch
    from bfp200 import _lib
    L = _lib.lib()
    buf = torch.zeros(4096, dtype=torch.int16, device="cuda")
    base = buf.data_ptr()
    for xm_off, wm_off, om_off in [(2, 0, 0), (0, 2, 0), (0, 0, 1)]:
        rc = L.bfp200_matvec_noalloc(base + xm_off, base, base + wm_off, base, 16, 16, 1, base + 64 + om_off,
                                     base + 128, None)
        assert rc == _lib.EINVAL and "aligned" in _lib.last_error()
    torch.cuda.synchronize()
