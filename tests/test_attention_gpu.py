"""Pyramid causal attention kernel vs an fp32 PyTorch restatement."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v):
    """q [B, ql, H, d], k/v [B, kl, H, d] fp32 -> [B, ql, H, d] (bottom-right causal)."""
    B, ql, H, d = q.shape
    kl = k.shape[1]
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(d)
    qi = torch.arange(ql, device=q.device)[:, None] + (kl - ql)
    ki = torch.arange(kl, device=q.device)[None, :]
    s = s.masked_fill(ki > qi, float("-inf"))
    return torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), v)


@pytest.mark.parametrize("d", [32, 64])
@pytest.mark.parametrize("ql,kl", [(912, 912), (786, 912), (32, 158), (1, 70), (200, 200), (130, 257), (64, 64)])
def test_fmha_fused_qkv_fwd_bwd(d, ql, kl):
    from primus_dlrm_b200.ops.attention import pyramid_attention_qkv
    torch.manual_seed(ql * 7 + kl + d)
    B, H = 3, 4
    qkv = torch.randn(B, kl, 3, H, d, device="cuda").to(torch.bfloat16).requires_grad_(True)
    o = pyramid_attention_qkv(qkv, ql)
    x = qkv.detach().float().requires_grad_(True)
    r = _ref(x[:, kl - ql:, 0], x[:, :, 1], x[:, :, 2])
    torch.testing.assert_close(o.float(), r, rtol=2e-2, atol=2e-2)
    do = torch.randn_like(r)
    o.backward(do.to(torch.bfloat16))
    r.backward(do.to(torch.bfloat16).float())
    g, gr = qkv.grad.float(), x.grad
    for part in range(3):
        err = (g[:, :, part] - gr[:, :, part]).abs().max().item()
        scale = gr[:, :, part].abs().max().item() + 1e-6
        assert err / scale < 3e-2, f"part {part}: max err {err} (scale {scale})"
    assert torch.all(g[:, : kl - ql, 0] == 0), "pruned query rows must get zero gradient"


def test_fmha_layout_strided_views():
    """Separate strided q/k/v views (not from one buffer) go through the same kernels."""
    from primus_dlrm_b200.ops.attention import _NativeFMHA
    B, H, d, kl, ql = 2, 8, 32, 300, 100
    big = torch.randn(B, kl, 5, H, d, device="cuda").to(torch.bfloat16)
    q = big[:, kl - ql:, 0].requires_grad_(False)
    k, v = big[:, :, 2], big[:, :, 4]
    o = _NativeFMHA.apply(q, k, v, d ** -0.5)
    r = _ref(q.float(), k.float(), v.float())
    torch.testing.assert_close(o.float(), r, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("d", [32, 64])
@pytest.mark.parametrize("ql,kl", [(912, 912), (786, 912), (32, 158), (1, 70), (200, 200), (130, 257), (129, 129)])
def test_fmha_tc_fwd_matches_reference(d, ql, kl):
    """tcgen05 forward (TMA + TMEM) vs fp32 attention; LSE in the log2 domain."""
    from primus_dlrm_b200.ops import _ext
    G = _ext.gemm()
    torch.manual_seed(ql + 3 * kl + d)
    B, H = 3, 4
    qkv = (2.0 * torch.randn(B, kl, 3, H, d, device="cuda")).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, lse = G.fmha_fwd_tc(qkv, ql, d ** -0.5, err)
    x = qkv.float()
    r = _ref(x[:, kl - ql:, 0], x[:, :, 1], x[:, :, 2])
    assert int(err.item()) == 0
    torch.testing.assert_close(o.float(), r, rtol=2e-2, atol=2e-2)
    q, k = x[:, kl - ql:, 0], x[:, :, 1]
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(d)
    qi = torch.arange(ql, device="cuda")[:, None] + (kl - ql)
    s = s.masked_fill(torch.arange(kl, device="cuda")[None, :] > qi, float("-inf"))
    lse_ref = torch.logsumexp(s, -1) / math.log(2.0)
    torch.testing.assert_close(lse, lse_ref, rtol=1e-3, atol=1e-2)


def test_fmha_tc_large_logits_rescale():
    """Rows whose running max grows across key tiles exercise the O rescale."""
    from primus_dlrm_b200.ops import _ext
    G = _ext.gemm()
    B, H, d, kl = 2, 2, 32, 400
    torch.manual_seed(0)
    qkv = torch.randn(B, kl, 3, H, d, device="cuda")
    qkv[:, :, 1] *= torch.linspace(0.1, 6.0, kl, device="cuda")[None, :, None, None]   # growing logits
    qkv = qkv.to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, _ = G.fmha_fwd_tc(qkv, kl, d ** -0.5, err)
    x = qkv.float()
    torch.testing.assert_close(o.float(), _ref(x[:, :, 0], x[:, :, 1], x[:, :, 2]), rtol=2e-2, atol=2e-2)


def test_fmha_tc_fwd_vs_reference_pyramid_v6_shapes():
    """Every layer shape of the v6 pyramid (d = 32, 8 heads), small batch."""
    from primus_dlrm_b200.ops import _ext
    G = _ext.gemm()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for ql, kl in [(912, 912), (661, 786), (409, 535), (158, 283), (32, 158)]:
        qkv = torch.randn(2, kl, 3, 8, 32, device="cuda").to(torch.bfloat16)
        o, _ = G.fmha_fwd_tc(qkv, ql, 32 ** -0.5, err)
        x = qkv.float()
        torch.testing.assert_close(o.float(), _ref(x[:, kl - ql:, 0], x[:, :, 1], x[:, :, 2]), rtol=2e-2, atol=2e-2)
    assert int(err.item()) == 0


@pytest.mark.parametrize("ql,kl", [(912, 912), (786, 912), (32, 158), (1, 70), (200, 200), (130, 257), (129, 129),
                                   (409, 535), (960, 1000)])
def test_fmha_tc_bwd_matches_reference(ql, kl):
    """tcgen05 backward (d = 32) vs autograd of the fp32 restatement."""
    from primus_dlrm_b200.ops import _ext
    G = _ext.gemm()
    torch.manual_seed(ql * 5 + kl)
    B, H, d = 2, 3, 32
    qkv = torch.randn(B, kl, 3, H, d, device="cuda").to(torch.bfloat16)
    q, k, v = qkv[:, kl - ql:, 0], qkv[:, :, 1], qkv[:, :, 2]
    o, lse = G.fmha_fwd(q, k, v, d ** -0.5)
    do = torch.randn(B, ql, H, d, device="cuda").to(torch.bfloat16)
    dqkv = torch.full_like(qkv, float("nan"))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    G.fmha_bwd_tc(qkv, o, lse, do, dqkv, ql, d ** -0.5, err)
    assert int(err.item()) == 0
    x = qkv.float().requires_grad_(True)
    r = _ref(x[:, kl - ql:, 0], x[:, :, 1], x[:, :, 2])
    r.backward(do.float())
    g = dqkv.float()
    assert torch.isfinite(g).all(), "every element of dqkv must be written"
    for part in range(3):
        e = (g[:, :, part] - x.grad[:, :, part]).abs().max().item()
        sc = x.grad[:, :, part].abs().max().item() + 1e-6
        assert e / sc < 3e-2, f"part {part}: max err {e} (scale {sc})"
    assert torch.all(g[:, : kl - ql, 0] == 0)


@pytest.mark.parametrize("warps", [4, 8])
@pytest.mark.parametrize("ql,kl", [(912, 912), (158, 283), (1, 70), (130, 257)])
def test_fmha_fwd_cta_sizes_match_reference(warps, ql, kl):
    """Both CTA sizes of the mma.sync forward (64- and 128-query CTAs, d = 32)."""
    from primus_dlrm_b200.ops import _ext
    G = _ext.gemm()
    torch.manual_seed(ql + kl + warps)
    B, H, d = 2, 4, 32
    qkv = torch.randn(B, kl, 3, H, d, device="cuda").to(torch.bfloat16)
    q, k, v = qkv[:, kl - ql:, 0], qkv[:, :, 1], qkv[:, :, 2]
    o, lse = G.fmha_fwd(q, k, v, d ** -0.5, warps)
    x = qkv.float()
    torch.testing.assert_close(o.float(), _ref(x[:, kl - ql:, 0], x[:, :, 1], x[:, :, 2]), rtol=2e-2, atol=2e-2)
