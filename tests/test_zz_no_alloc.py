"""The allocation-free sparse-update entry point (``pd_emb_sparse_update_noalloc``).

Some callers cannot let this library allocate device memory while they run
(a host runtime with a fixed memory budget, or a latency-critical thread that
must not block on the allocator). For them the library exports one C entry
point that takes its scratch from a fixed array compiled into the library.
This test calls that exported C symbol through ctypes and checks it against
the regular entry point (``_C.emb_reduce_update``) on the same inputs, for two
calls in a row, within the tolerance the other kernel tests use.

The file name sorts last so that a run which stops at the first failure has
already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
OPT_CODES = {"sgd": 0, "adagrad": 1, "row_wise_adagrad": 2, "adam": 3}


def _lib():
    import primus_dlrm_b200._C as C
    lib = ctypes.CDLL(C.__file__)
    fn = lib.pd_emb_sparse_update_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                   ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_void_p,
                   ctypes.c_void_p]
    return fn


def _state(kind, rows, dim):
    if kind == "sgd":
        return []
    if kind == "adagrad":
        return [torch.zeros(rows, dim, device=DEV)]
    if kind == "row_wise_adagrad":
        return [torch.zeros(rows, device=DEV)]
    return [torch.zeros(rows, dim, device=DEV), torch.zeros(rows, dim, device=DEV)]


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


@pytest.mark.parametrize("kind", ["row_wise_adagrad", "adam", "sgd", "adagrad"])
@pytest.mark.parametrize("gdtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_regular_entry_point(kind, gdtype):
    from primus_dlrm_b200.ops import _ext
    C = _ext.core()
    fn = _lib()
    torch.manual_seed(0)
    rows, dim, n = 700, 128, 5000
    w0 = torch.randn(rows, dim, device=DEV)
    w_reg, w_na = w0.clone(), w0.clone()
    s_reg, s_na = _state(kind, rows, dim), _state(kind, rows, dim)
    err_reg = torch.zeros(1, dtype=torch.int32, device=DEV)
    err_na = torch.zeros(1, dtype=torch.int32, device=DEV)
    lr, eps, wd, b1, b2 = 0.05, 1e-6, 1e-3, 0.9, 0.999
    stream = torch.cuda.current_stream()
    for step in (1, 2):
        ids = torch.randint(0, rows, (n,), device=DEV)
        ids[:300] = 11          # a hot row whose run crosses many 32-id chunks (uses the scratch)
        grads = torch.randn(n, dim, device=DEV).to(gdtype)
        skeys, perm = torch.sort(ids)
        bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
        # regular entry point (one slot, one table)
        meta = torch.tensor([[0, 0, 0, -1, n]], dtype=torch.int64)
        tmeta = torch.tensor([[rows, rows, 0, 0, 1, dim]], dtype=torch.int64)
        ptrs = torch.tensor([w_reg.data_ptr()], dtype=torch.int64, device=DEV)
        s1 = s_reg[0] if len(s_reg) > 0 else w_reg.new_empty(0)
        s2 = s_reg[1] if len(s_reg) > 1 else w_reg.new_empty(0)
        C.emb_reduce_update([grads], meta, [w_reg], [ptrs], [s1], [s2], tmeta, dim, skeys, perm, None, None,
                            OPT_CODES[kind], lr, eps, wd, b1, b2, bc1, bc2, err_reg)
        # allocation-free entry point, called through its exported C symbol
        rc = fn(_ptr(skeys), _ptr(perm), n, _ptr(grads), 1 if gdtype == torch.bfloat16 else 0, dim,
                _ptr(w_na), rows, dim, _ptr(s_na[0] if len(s_na) > 0 else None),
                _ptr(s_na[1] if len(s_na) > 1 else None), OPT_CODES[kind], lr, eps, wd, b1, b2, bc1, bc2,
                _ptr(err_na), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, f"pd_emb_sparse_update_noalloc returned {rc}"
        torch.cuda.synchronize()
        torch.testing.assert_close(w_na, w_reg, rtol=1e-4, atol=1e-5)
        for a, b in zip(s_na, s_reg):
            torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5)
        assert int(err_na.item()) == 0 and int(err_reg.item()) == 0
    assert not torch.equal(w_na, w0)


def test_noalloc_rejects_oversized_inputs():
    fn = _lib()
    big = (1 << 18) + 1
    rc = fn(ctypes.c_void_p(16), ctypes.c_void_p(16), big, ctypes.c_void_p(16), 0, 128, ctypes.c_void_p(16),
            10, 128, ctypes.c_void_p(0), ctypes.c_void_p(0), 0, 0.1, 1e-8, 0.0, 0.9, 0.999, 1.0, 1.0,
            ctypes.c_void_p(0), ctypes.c_void_p(0))
    assert rc == -1
    rc = fn(ctypes.c_void_p(16), ctypes.c_void_p(16), 10, ctypes.c_void_p(16), 0, 512, ctypes.c_void_p(16),
            10, 512, ctypes.c_void_p(0), ctypes.c_void_p(0), 0, 0.1, 1e-8, 0.0, 0.9, 0.999, 1.0, 1.0,
            ctypes.c_void_p(0), ctypes.c_void_p(0))
    assert rc == -1


def _regular(C, grads, skeys, perm, w, state, kind, rows, dim, n, step, err, hp=(0.05, 1e-6, 1e-3, 0.9, 0.999)):
    lr, eps, wd, b1, b2 = hp
    meta = torch.tensor([[0, 0, 0, -1, n]], dtype=torch.int64)
    tmeta = torch.tensor([[rows, rows, 0, 0, 1, dim]], dtype=torch.int64)
    ptrs = torch.tensor([w.data_ptr()], dtype=torch.int64, device=DEV)
    s1 = state[0] if len(state) > 0 else w.new_empty(0)
    s2 = state[1] if len(state) > 1 else w.new_empty(0)
    C.emb_reduce_update([grads], meta, [w], [ptrs], [s1], [s2], tmeta, dim, skeys, perm, None, None,
                        OPT_CODES[kind], lr, eps, wd, b1, b2, 1 - b1 ** step, 1 - b2 ** step, err)


def _noalloc(fn, grads, skeys, perm, w, state, kind, rows, dim, n, step, err, grad_stride=None,
             hp=(0.05, 1e-6, 1e-3, 0.9, 0.999)):
    lr, eps, wd, b1, b2 = hp
    gs = grads.stride(0) if grad_stride is None else grad_stride
    return fn(_ptr(skeys), _ptr(perm), n, _ptr(grads), 1 if grads.dtype == torch.bfloat16 else 0, gs,
              _ptr(w), rows, dim, _ptr(state[0] if len(state) > 0 else None),
              _ptr(state[1] if len(state) > 1 else None), OPT_CODES[kind], lr, eps, wd, b1, b2,
              1 - b1 ** step, 1 - b2 ** step, _ptr(err), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("gdtype", [torch.bfloat16, torch.float32])
def test_noalloc_max_dim_strided_grads_and_full_scratch(gdtype):
    """dim = 256 (the maximum), a gradient view whose row stride exceeds dim,
    and n = the maximum id count, so every chunk of the fixed scratch is used."""
    from primus_dlrm_b200.ops import _ext
    C = _ext.core()
    fn = _lib()
    torch.manual_seed(1)
    rows, dim, n = 4096, 256, 1 << 18
    w0 = torch.randn(rows, dim, device=DEV)
    w_reg, w_na = w0.clone(), w0.clone()
    s_reg, s_na = _state("adam", rows, dim), _state("adam", rows, dim)
    e_reg = torch.zeros(1, dtype=torch.int32, device=DEV)
    e_na = torch.zeros(1, dtype=torch.int32, device=DEV)
    for step in (1, 2):
        ids = torch.randint(0, rows, (n,), device=DEV)
        ids[: n // 8] = 7           # one run across thousands of chunks
        ids[n // 8: n // 4] = 4095
        base = torch.randn(n, dim + 8, device=DEV).to(gdtype)
        grads = base[:, :dim]       # row stride dim + 8 elements
        skeys, perm = torch.sort(ids)
        _regular(C, grads, skeys, perm, w_reg, s_reg, "adam", rows, dim, n, step, e_reg)
        rc = _noalloc(fn, grads, skeys, perm, w_na, s_na, "adam", rows, dim, n, step, e_na)
        assert rc == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(w_na, w_reg, rtol=1e-4, atol=1e-4)
        for a, b in zip(s_na, s_reg):
            torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-4)
        assert int(e_na.item()) == 0 and int(e_reg.item()) == 0


def test_noalloc_out_of_range_ids_and_null_err():
    from primus_dlrm_b200.ops import _ext
    C = _ext.core()
    fn = _lib()
    torch.manual_seed(2)
    rows, dim, n = 500, 64, 3000
    w0 = torch.randn(rows, dim, device=DEV)
    # (a) a few ids >= rows: skipped, recorded as 1 in err, the other rows match the regular path
    ids = torch.randint(0, rows, (n,), device=DEV)
    ids[:5] = rows + 3
    grads = torch.randn(n, dim, device=DEV)
    skeys, perm = torch.sort(ids)
    w_reg, w_na = w0.clone(), w0.clone()
    s_reg, s_na = _state("row_wise_adagrad", rows, dim), _state("row_wise_adagrad", rows, dim)
    e_reg = torch.zeros(1, dtype=torch.int32, device=DEV)
    e_na = torch.zeros(1, dtype=torch.int32, device=DEV)
    _regular(C, grads, skeys, perm, w_reg, s_reg, "row_wise_adagrad", rows, dim, n, 1, e_reg)
    assert _noalloc(fn, grads, skeys, perm, w_na, s_na, "row_wise_adagrad", rows, dim, n, 1, e_na) == 0
    torch.cuda.synchronize()
    assert int(e_na.item()) == 1
    torch.testing.assert_close(w_na, w_reg, rtol=1e-4, atol=1e-5)
    # (b) a perm value outside [0, n): skipped and recorded
    perm_bad = perm.clone()
    perm_bad[0] = n + 11
    e_na.zero_()
    assert _noalloc(fn, grads, skeys, perm_bad, w0.clone(), _state("sgd", rows, dim), "sgd", rows, dim, n, 1,
                    e_na) == 0
    torch.cuda.synchronize()
    assert int(e_na.item()) == 1
    # (c) err = NULL: the call runs and matches the regular path
    ids = torch.randint(0, rows, (n,), device=DEV)
    skeys, perm = torch.sort(ids)
    w_reg, w_na = w0.clone(), w0.clone()
    e_reg.zero_()
    _regular(C, grads, skeys, perm, w_reg, [], "sgd", rows, dim, n, 1, e_reg)
    assert _noalloc(fn, grads, skeys, perm, w_na, [], "sgd", rows, dim, n, 1, None) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(w_na, w_reg, rtol=1e-5, atol=1e-6)


def test_noalloc_rejects_bad_arguments():
    fn = _lib()
    rows, dim, n = 64, 32, 100
    w = torch.zeros(rows, dim, device=DEV)
    m = torch.zeros(rows, dim, device=DEV)
    grads = torch.zeros(n, dim + 4, device=DEV)
    ids = torch.zeros(n, dtype=torch.int64, device=DEV)
    perm = torch.arange(n, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call(grads_p=None, gs=dim + 4, w_p=None, d=dim, s1=None, s2=None, kind=3):
        return fn(_ptr(ids), _ptr(perm), n, grads_p if grads_p is not None else _ptr(grads), 0, gs,
                  w_p if w_p is not None else _ptr(w), rows, d, s1 if s1 is not None else _ptr(m),
                  s2 if s2 is not None else _ptr(m), kind, 0.1, 1e-8, 0.0, 0.9, 0.999, 1.0, 1.0, _ptr(err), st)

    assert call(d=30, gs=32) == -2                                      # dim % 4 != 0
    assert call(w_p=ctypes.c_void_p(0)) == -2                           # null weight
    assert call(s2=ctypes.c_void_p(0)) == -2                            # Adam without its second moment
    assert call(gs=dim - 4) == -2                                       # row stride below dim
    assert call(gs=dim + 2) == -2                                       # row stride not a multiple of 4
    assert call(grads_p=ctypes.c_void_p(grads.data_ptr() + 4)) == -2    # misaligned gradient rows
    assert call(w_p=ctypes.c_void_p(w.data_ptr() + 8)) == -2            # misaligned table
    torch.cuda.synchronize()
    assert int(err.item()) == 0                                         # nothing was launched
