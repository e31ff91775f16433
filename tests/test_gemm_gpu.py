"""tcgen05 GEMM (sm_100a) vs fp32 PyTorch matmul, incl. strided batched views
and the fused epilogues."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _bf(*s):
    return torch.randn(*s, device="cuda").to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(1000, 768, 256), (128, 256, 1024), (129, 128, 64), (4099, 1024, 256),
                                   (77, 64, 192), (2048, 256, 512)])
def test_plain(M, N, K):
    from primus_dlrm_b200.ops.dense import tc_gemm, gemm_error_code
    a, b = _bf(1, M, K), _bf(1, N, K)
    c = torch.empty(1, M, N, device="cuda", dtype=torch.bfloat16)
    tc_gemm(a, b, c)
    ref = a.float() @ b.float().transpose(1, 2)
    torch.testing.assert_close(c.float(), ref, rtol=2e-2, atol=2e-2 * K ** 0.5)
    assert gemm_error_code("cuda") == 0


@pytest.mark.parametrize("M,N,K", [(1000, 256, 768), (129, 1024, 256), (300, 256, 1024), (77, 64, 200)])
def test_b_transposed_in_place(M, N, K):
    """B given as a stored weight [K, N] (N contiguous), read MN-major: C = A @ W."""
    from primus_dlrm_b200.ops.dense import tc_gemm, gemm_error_code
    a, w = _bf(1, M, K), _bf(1, K, N)
    c = torch.empty(1, M, N, device="cuda", dtype=torch.bfloat16)
    tc_gemm(a, w, c, b_kn=True)
    ref = a.float() @ w.float()
    torch.testing.assert_close(c.float(), ref, rtol=2e-2, atol=2e-2 * K ** 0.5)
    assert gemm_error_code("cuda") == 0


def test_b_transposed_batched_ns_layout():
    """Per-NS-token weights [T, K, N] applied transposed to strided NS rows."""
    from primus_dlrm_b200.ops.dense import tc_gemm
    Bsz, T, n_s, K, N = 300, 40, 24, 768, 256
    x = _bf(Bsz, T, K)
    w = _bf(T - n_s, K, N)
    y = torch.zeros(Bsz, T, N, device="cuda", dtype=torch.bfloat16)
    tc_gemm(x[:, n_s:].transpose(0, 1), w, y[:, n_s:].transpose(0, 1), b_kn=True)
    ref = torch.einsum("btk,tkn->btn", x[:, n_s:].float(), w.float())
    torch.testing.assert_close(y[:, n_s:].float(), ref, rtol=2e-2, atol=0.6)
    assert torch.all(y[:, :n_s] == 0)


@pytest.mark.parametrize("rows,M,N", [(5000, 768, 256), (1000, 256, 1024), (777, 128, 384), (64, 64, 64)])
def test_wgrad_split_k(rows, M, N):
    """C = A^T B over the rows (weight gradient), both operands as stored."""
    from primus_dlrm_b200.ops.dense import gemm_error_code, tc_wgrad
    a, b = _bf(1, rows, M), _bf(1, rows, N)
    c = tc_wgrad(a, b, torch.zeros(1, M, N, device="cuda"))
    ref = a[0].float().t() @ b[0].float()
    torch.testing.assert_close(c[0], ref, rtol=1e-3, atol=1e-3 * rows ** 0.5)
    assert gemm_error_code("cuda") == 0


def test_wgrad_per_token_strided():
    """Per-NS-token weight gradients over strided views (one batch per token)."""
    from primus_dlrm_b200.ops.dense import tc_wgrad
    Bsz, T, n_s, M, N = 600, 40, 24, 256, 768
    dy, x = _bf(Bsz, T, M), _bf(Bsz, T, N)
    c = tc_wgrad(dy[:, n_s:].transpose(0, 1), x[:, n_s:].transpose(0, 1), torch.zeros(T - n_s, M, N, device="cuda"))
    ref = torch.einsum("btm,btn->tmn", dy[:, n_s:].float(), x[:, n_s:].float())
    torch.testing.assert_close(c, ref, rtol=1e-3, atol=1e-3 * Bsz ** 0.5)


def test_wgrad_sum_over_samples():
    """One weight gradient summed over the samples of a strided token range."""
    from primus_dlrm_b200.ops.dense import tc_wgrad
    Bsz, T, off, L, M, N = 300, 100, 20, 64, 256, 256
    dx, h = _bf(Bsz, T, M), _bf(Bsz, L, N)
    c = tc_wgrad(dx[:, off:off + L], h, torch.zeros(1, M, N, device="cuda"), l_sum=True)
    ref = torch.einsum("blm,bln->mn", dx[:, off:off + L].float(), h.float())
    torch.testing.assert_close(c[0], ref, rtol=1e-3, atol=1e-3 * (Bsz * L) ** 0.5)


def test_batched_strided_ns_layout():
    """NS rows of every sample as one batch per token (row stride T*K, batch stride K)."""
    from primus_dlrm_b200.ops.dense import tc_gemm
    Bsz, T, n_s, K, N = 300, 40, 24, 256, 768
    x = _bf(Bsz, T, K)
    w = _bf(T - n_s, N, K)
    y = torch.zeros(Bsz, T, N, device="cuda", dtype=torch.bfloat16)
    tc_gemm(x[:, n_s:].transpose(0, 1), w, y[:, n_s:].transpose(0, 1))
    ref = torch.einsum("btk,tnk->btn", x[:, n_s:].float(), w.float())
    torch.testing.assert_close(y[:, n_s:].float(), ref, rtol=2e-2, atol=0.35)
    assert torch.all(y[:, :n_s] == 0)


def test_epilogues():
    from primus_dlrm_b200.ops.dense import tc_gemm
    M, N, K = 700, 256, 256
    a, b = _bf(1, M, K), _bf(1, N, K)
    acc = a.float() @ b.float().transpose(1, 2)
    pre_b = acc.to(torch.bfloat16)
    c = torch.empty(1, M, N, device="cuda", dtype=torch.bfloat16)
    aux = torch.empty_like(c)
    tc_gemm(a, b, c, "gelu", AUX=aux)
    torch.testing.assert_close(aux.float(), pre_b.float(), rtol=2e-2, atol=0.3)
    torch.testing.assert_close(c.float(), F.gelu(aux.float()), rtol=2e-2, atol=2e-2)
    r = _bf(1, M, N)
    tc_gemm(a, b, c, "residual", R=r)
    torch.testing.assert_close(c.float(), acc + r.float(), rtol=2e-2, atol=0.35)
    tc_gemm(a, b, c, "dgelu", R=r)
    x = r.float().requires_grad_(True)
    F.gelu(x).backward(torch.ones_like(x))
    torch.testing.assert_close(c.float(), acc * x.grad, rtol=3e-2, atol=0.5)


def test_gelu_derivative_store_and_product_epilogues():
    """gelu_d: C = GELU(x), AUX = GELU'(x) for the fp32 x = acc; mul: C = acc * R.
    Against fp32 autograd of torch's exact-erf GELU."""
    from primus_dlrm_b200.ops.dense import tc_gemm
    M, N, K = 700, 256, 128
    a, b = _bf(1, M, K), _bf(1, N, K)
    acc = a.float() @ b.float().transpose(1, 2)
    c = torch.empty(1, M, N, device="cuda", dtype=torch.bfloat16)
    d = torch.empty_like(c)
    tc_gemm(a, b, c, "gelu_d", AUX=d)
    x = acc.to(torch.bfloat16).float().requires_grad_(True)
    y = F.gelu(x)
    y.backward(torch.ones_like(y))
    torch.testing.assert_close(c.float(), y.detach(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(d.float(), x.grad, rtol=2e-2, atol=2e-2)
    # with an addend (bias broadcast through zero strides) before the activation
    bias = (torch.randn(N, device="cuda") * 0.5).to(torch.bfloat16)
    tc_gemm(a, b, c, "gelu_d", R=bias.view(1, 1, N).expand(1, M, N), AUX=d)
    x2 = (acc + bias.float()).to(torch.bfloat16).float().requires_grad_(True)
    F.gelu(x2).backward(torch.ones_like(x2))
    torch.testing.assert_close(d.float(), x2.grad, rtol=2e-2, atol=2e-2)
    r = _bf(1, M, N)
    tc_gemm(a, b, c, "mul", R=r)
    torch.testing.assert_close(c.float(), acc * r.float(), rtol=2e-2, atol=0.5)


def test_mixed_linear_and_ffn_match_torch_path():
    import os

    from primus_dlrm_b200.ops import dense
    torch.manual_seed(0)
    Bsz, T, n_s, D, F_ = 64, 40, 24, 256, 1024
    x = (_bf(Bsz, T, D) * 0.5).requires_grad_(True)
    z = _bf(Bsz, T, D).requires_grad_(True)
    w1 = (torch.randn(F_, D, device="cuda") * 0.05).requires_grad_(True)
    w2 = (torch.randn(D, F_, device="cuda") * 0.05).requires_grad_(True)
    wn1 = (torch.randn(T - n_s, F_, D, device="cuda") * 0.05).requires_grad_(True)
    wn2 = (torch.randn(T - n_s, D, F_, device="cuda") * 0.05).requires_grad_(True)
    out = dense.mixed_ffn(x, z, n_s, w1, w2, wn1, wn2)
    assert out is not None
    g = torch.randn_like(out)
    out.backward(g)
    got = [t.grad.clone() for t in (x, z, w1, w2, wn1, wn2)]
    for t in (x, z, w1, w2, wn1, wn2):
        t.grad = None
    h = dense._MixedLinearTorch.apply(x, w1, wn1, n_s, "gelu")
    ref = z + dense._MixedLinearTorch.apply(h, w2, wn2, n_s, "")
    torch.testing.assert_close(out.float(), ref.float(), rtol=3e-2, atol=3e-2)
    ref.backward(g)
    for a, b in zip(got, (x.grad, z.grad, w1.grad, w2.grad, wn1.grad, wn2.grad)):
        torch.testing.assert_close(a.float(), b.float(), rtol=5e-2, atol=5e-2 * (b.float().abs().max().item() + 1e-3))


def test_gelu_epilogue_accuracy_vs_exact_erf():
    """The GEMM's GELU / GELU' (division-free polynomial normal CDF) against
    torch's exact erf GELU, on a grid of pre-activations in [-8, 8]: within one
    bf16 rounding of the exact value."""
    from primus_dlrm_b200.ops.dense import tc_gemm
    M, N, K = 256, 256, 64
    # A = identity-like rows so the accumulator equals a chosen value per column
    vals = torch.linspace(-8, 8, N, device="cuda")
    a = torch.zeros(1, M, K, device="cuda")
    a[0, :, 0] = 1.0
    b = torch.zeros(1, N, K, device="cuda")
    b[0, :, 0] = vals
    a, b = a.to(torch.bfloat16), b.to(torch.bfloat16)
    c = torch.empty(1, M, N, device="cuda", dtype=torch.bfloat16)
    tc_gemm(a, b, c, "gelu")
    x = b[0, :, 0].float()
    ref = F.gelu(x)
    torch.testing.assert_close(c[0, 0].float(), ref.to(torch.bfloat16).float(), rtol=0, atol=1e-2)
    r = x.to(torch.bfloat16).expand(1, M, N).contiguous()
    ones = torch.zeros(1, N, K, device="cuda")
    ones[0, :, 0] = 1.0
    tc_gemm(a, ones.to(torch.bfloat16), c, "dgelu", R=r)
    xg = x.clone().requires_grad_(True)
    F.gelu(xg).backward(torch.ones_like(xg))
    torch.testing.assert_close(c[0, 0].float(), xg.grad.to(torch.bfloat16).float(), rtol=0, atol=1e-2)


def test_gemm_bias_addend_before_gelu():
    """R broadcast through zero strides is added before the activation."""
    from primus_dlrm_b200.ops.dense import tc_gemm
    torch.manual_seed(3)
    M, N, K = 1000, 256, 384
    A = torch.randn(1, M, K, device="cuda").to(torch.bfloat16)
    W = (torch.randn(1, N, K, device="cuda") / K ** 0.5).to(torch.bfloat16)
    b = torch.randn(N, device="cuda").to(torch.bfloat16)
    C = torch.empty(1, M, N, dtype=torch.bfloat16, device="cuda")
    pre = torch.empty_like(C)
    tc_gemm(A, W, C, "gelu", R=b.reshape(1, 1, N).expand(1, M, N), AUX=pre)
    ref_pre = A.float()[0] @ W.float()[0].t() + b.float()
    torch.testing.assert_close(pre.float()[0], ref_pre, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(C.float()[0], torch.nn.functional.gelu(ref_pre), rtol=2e-2, atol=2e-2)


def test_tokenizer_mlp_native_matches_torch():
    """Fused tokenizer MLP (bias + GELU, bias + positional addend) fwd / bwd vs fp32."""
    from primus_dlrm_b200.ops.dense import mlp2
    torch.manual_seed(4)
    B, L, K, D = 16, 40, 384, 256
    l1 = torch.nn.Linear(K, D).cuda()
    l2 = torch.nn.Linear(D, D).cuda()
    pos = torch.nn.Parameter(torch.randn(64, D, device="cuda") * 0.1)
    x = torch.randn(B, L, K, device="cuda").to(torch.bfloat16).requires_grad_(True)
    y = mlp2(x, l1, l2, addend=pos[:L])
    assert y.dtype == torch.bfloat16
    g = torch.randn_like(y)
    y.backward(g)
    grads = [t.grad.clone() for t in (l1.weight, l1.bias, l2.weight, l2.bias, pos)] + [x.grad.float().clone()]
    for t in (l1.weight, l1.bias, l2.weight, l2.bias, pos):
        t.grad = None
    xr = x.detach().float().requires_grad_(True)
    yr = l2(torch.nn.functional.gelu(l1(xr))) + pos[:L]
    torch.testing.assert_close(y.float(), yr, rtol=3e-2, atol=3e-2)
    yr.backward(g.float())
    ref = [t.grad for t in (l1.weight, l1.bias, l2.weight, l2.bias, pos)] + [xr.grad]
    for got, exp in zip(grads, ref):
        err = (got.float() - exp).abs().max().item()
        assert err / (exp.abs().max().item() + 1e-6) < 3e-2


def test_tokenizer_mlp_backward_reads_strided_gradient_in_place():
    """The tokenizer MLP's backward with its output gradient as a token range
    of a wider [B, T, N] buffer (what the concatenation of the S pools hands
    it) against the same gradient made contiguous."""
    from primus_dlrm_b200.ops import dense
    torch.manual_seed(5)
    Bsz, L, T, K, N = 96, 128, 320, 384, 256
    l1 = torch.nn.Linear(K, N, device="cuda")
    l2 = torch.nn.Linear(N, N, device="cuda")
    pos = (torch.randn(L, N, device="cuda") * 0.1).requires_grad_(True)
    x = (_bf(Bsz, L, K) * 0.5).requires_grad_(True)
    G = _bf(Bsz, T, N)
    grads = []
    for strided in (True, False):
        for t in (x, pos, l1.weight, l1.bias, l2.weight, l2.bias):
            t.grad = None
        y = dense.mlp2(x, l1, l2, addend=pos)
        dout = G[:, 64:64 + L]
        assert not dout.is_contiguous()
        y.backward(dout if strided else dout.contiguous())
        grads.append([t.grad.float().clone() for t in (x, pos, l1.weight, l1.bias, l2.weight, l2.bias)])
    for name, a, b in zip(["x", "pos", "w1", "b1", "w2", "b2"], *grads):
        torch.testing.assert_close(a, b, rtol=1e-2, atol=1e-2 * (b.abs().max().item() + 1e-3), msg=name)
