"""The no-allocation entry point ng_rms_mod_bwd_noalloc (csrc/noalloc.h), called through its exported C symbol, against
the regular allocating entry point of the same backward. It is for callers that cannot allocate device memory when
they call (under a fixed memory pool, in an allocation-free loop, or from plain C without PyTorch's allocator).

This file is collected last on purpose: if it fails, a run that stops at the first failure has run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

c_void_p, c_int64, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int


def _lib():
    import nano_gpic_b200._C as C
    lib = ctypes.CDLL(C.__file__)
    f = lib.ng_rms_mod_bwd_noalloc
    f.restype = c_int
    f.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                  c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_void_p]
    e = lib.ng_noalloc_error_string
    e.restype = ctypes.c_char_p
    e.argtypes = [c_int]
    return f, e


def _ptr(t):
    return None if t is None else t.data_ptr()


def _close(a, b, rtol=2e-2, atol=2e-2, what=""):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= atol + rtol * ref, f"{what}: max err {err} vs ref max {ref}"


def _case(M, C, rpg, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    G = M // rpg
    dh = torch.randn(M, C, device="cuda", generator=g).bfloat16()
    x = torch.randn(M, C, device="cuda", generator=g).bfloat16()
    dres = torch.randn(M, C, device="cuda", generator=g).bfloat16()
    w = torch.rand(C, device="cuda", generator=g) + 0.5
    mod = (torch.randn(G, 6 * C, device="cuda", generator=g) * 0.3).bfloat16()
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6)
    return dh, x, dres, w, mod, rstd


def test_noalloc_matches_allocating_entry_point_twice():
    from nano_gpic_b200._ext import ext
    f, err_str = _lib()
    stream = torch.cuda.current_stream()
    # two calls in a row, the second smaller than the first: the shared scratch still holds the first call's sums
    for (M, C, rpg, seed) in [(128 * 256 // 8, 1024, 256, 1), (40 * 56, 768, 56, 2)]:
        dh, x, dres, w, mod, rstd = _case(M, C, rpg, seed)
        G = M // rpg
        scale = mod[:, C:2 * C]
        # the existing (allocating) entry point
        dx_ref = torch.empty_like(x)
        dw_ref = torch.full((C,), 0.25, device="cuda")
        dmod_ref = torch.zeros(G, 6 * C, device="cuda")
        ext().rms_mod_bwd(dh, x, rstd, w, scale, dres, dx_ref, dw_ref, dmod_ref[:, :C], dmod_ref[:, C:2 * C], rpg,
                          None, 0)
        # the no-allocation entry point, same inputs, outputs pre-filled with garbage where they are overwritten
        dx = torch.full_like(x, 7.0)
        dw = torch.full((C,), 0.25, device="cuda")
        dmod = torch.full((G, 6 * C), -3.0, device="cuda")
        torch.cuda.synchronize()
        before = torch.cuda.memory_allocated()
        rc = f(_ptr(dh), _ptr(x), _ptr(rstd), _ptr(w), _ptr(scale), scale.stride(0), _ptr(dres), _ptr(dx), _ptr(dw),
               _ptr(dmod[:, :C]), dmod.stride(0), _ptr(dmod[:, C:2 * C]), dmod.stride(0), M, C, rpg,
               stream.cuda_stream)
        assert rc == 0, err_str(rc).decode()
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == before  # nothing went through PyTorch's allocator
        _close(dx, dx_ref, what="dx")
        _close(dw, dw_ref, rtol=1e-2, atol=1e-2, what="dw")
        _close(dmod[:, :2 * C], dmod_ref[:, :2 * C], rtol=1e-2, atol=1e-2, what="dshift/dscale")
        assert (dmod[:, 2 * C:] == -3.0).all()  # columns it does not own stay untouched


def test_noalloc_plain_rmsnorm_and_optional_outputs():
    """The plain-RMSNorm form (no modulation: one group of all rows) without a residual gradient, and the modulated
    form without a weight gradient, each twice in a row; M is not a multiple of the 64-row chunk, so the last chunk of
    every group is partial."""
    from nano_gpic_b200._ext import ext
    f, err_str = _lib()
    stream = torch.cuda.current_stream()
    for rep in range(2):
        # plain RMSNorm: scale = None, dres = None, dshift / dscale ignored
        M, C = 1000 + 37 * rep, 512
        dh, x, _, w, _, rstd = _case(M, C, M, 10 + rep)
        dx_ref, dw_ref = torch.empty_like(x), torch.zeros(C, device="cuda")
        ext().rms_mod_bwd(dh, x, rstd, w, None, None, dx_ref, dw_ref, None, None, 1, None, 0)
        dx, dw = torch.full_like(x, 5.0), torch.zeros(C, device="cuda")
        rc = f(_ptr(dh), _ptr(x), _ptr(rstd), _ptr(w), None, 0, None, _ptr(dx), _ptr(dw), None, 0, None, 0, M, C, 0,
               stream.cuda_stream)
        assert rc == 0, err_str(rc).decode()
        _close(dx, dx_ref, what="plain dx")
        _close(dw, dw_ref, rtol=1e-2, atol=1e-2, what="plain dw")
        # modulated, dw = None, groups of 100 rows (two chunks, the second partial)
        M, C, rpg = 700, 256, 100
        dh, x, dres, w, mod, rstd = _case(M, C, rpg, 20 + rep)
        G = M // rpg
        scale = mod[:, C:2 * C]
        dx_ref, dmod_ref = torch.empty_like(x), torch.zeros(G, 6 * C, device="cuda")
        ext().rms_mod_bwd(dh, x, rstd, w, scale, dres, dx_ref, None, dmod_ref[:, :C], dmod_ref[:, C:2 * C], rpg,
                          None, 0)
        dx, dmod = torch.full_like(x, 5.0), torch.full((G, 6 * C), 9.0, device="cuda")
        rc = f(_ptr(dh), _ptr(x), _ptr(rstd), _ptr(w), _ptr(scale), scale.stride(0), _ptr(dres), _ptr(dx), None,
               _ptr(dmod[:, :C]), dmod.stride(0), _ptr(dmod[:, C:2 * C]), dmod.stride(0), M, C, rpg,
               stream.cuda_stream)
        assert rc == 0, err_str(rc).decode()
        _close(dx, dx_ref, what="mod dx")
        _close(dmod[:, :2 * C], dmod_ref[:, :2 * C], rtol=1e-2, atol=1e-2, what="mod dshift/dscale")
    torch.cuda.synchronize()


def test_noalloc_rejects_oversized_call():
    f, err_str = _lib()
    C, rpg = 1024, 256
    M = 4096 * rpg  # 4096 groups x 4 chunks x 3 x 1024 values: far above the 2M-value scratch
    x = torch.empty(1, device="cuda")
    rc = f(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 6 * C, None, x.data_ptr(), None,
           None, 0, None, 0, M, C, rpg, torch.cuda.current_stream().cuda_stream)
    assert rc == 1 and b"NG_NOALLOC_RMS_SCRATCH_FLOATS" in err_str(rc)
    # more groups than a grid dimension holds: an argument error, nothing launched
    rc = f(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 48, None, x.data_ptr(), None,
           None, 0, None, 0, 70000, 8, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == 2 and b"65535" in err_str(rc)
