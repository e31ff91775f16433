"""DLRM kernels on the tcgen05 GEMM against fp32 PyTorch restatements:
the Linear / ReLU chain (bias + ReLU epilogues, ReLU mask in the backward's
data-gradient epilogue) and the fused low-rank DCNv2 cross layer."""
import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


@pytest.mark.parametrize("dims,final_act", [([13, 512, 256, 128], True), ([3456, 1024, 1024, 512, 256], True),
                                            ([3712, 256], False), ([192, 128, 64], True)])
def test_mlp_chain_matches_fp32(dims, final_act):
    """Forward against fp32 layer by layer; backward against an fp32
    restatement that takes the ReLU masks from the native forward (a bf16
    pre-activation within rounding of zero may take the other side of the
    ReLU than the fp32 one, which is rounding, not a kernel error)."""
    from primus_dlrm_b200.models.interaction import make_mlp
    from primus_dlrm_b200.ops.mlp import mlp_chain
    torch.manual_seed(len(dims) + dims[0])
    seq = make_mlp(dims, dropout=0.0, final_activation=final_act).to(DEV)
    lins = [m for m in seq if isinstance(m, nn.Linear)]
    relu = [final_act or i < len(lins) - 1 for i in range(len(lins))]
    B = 1000
    xb = torch.randn(B, dims[0], device=DEV).to(torch.bfloat16).requires_grad_(True)
    # native activations of every prefix of the chain (deterministic kernels)
    hs = [xb.detach().float()]
    with torch.no_grad():
        for n in range(1, len(lins) + 1):
            hs.append(mlp_chain(seq[: 2 * n if final_act or n < len(lins) else 2 * n - 1], xb.detach()).float())
    for n in range(len(lins)):          # each layer's forward against fp32 on the same input
        ref = hs[n] @ lins[n].weight.t() + lins[n].bias
        ref = torch.relu(ref) if relu[n] else ref
        assert _rel(hs[n + 1], ref) < 2e-2, n
    y = mlp_chain(seq, xb)
    dy = torch.randn_like(y.float()).to(torch.bfloat16)
    y.backward(dy)
    d = dy.float()
    ref_g = {}
    for n in reversed(range(len(lins))):
        if relu[n]:
            d = d * (hs[n + 1] > 0)
        ref_g[n] = (d.t() @ hs[n], d.sum(0))
        d = d @ lins[n].weight
    assert _rel(xb.grad, d) < 3e-2
    for n, lin in enumerate(lins):
        assert _rel(lin.weight.grad, ref_g[n][0]) < 3e-2, f"layer {n} weight"
        assert _rel(lin.bias.grad, ref_g[n][1]) < 3e-2, f"layer {n} bias"


@pytest.mark.parametrize("B,d,r", [(1000, 3456, 512), (257, 256, 64)])
def test_cross_layer_matches_fp32(B, d, r):
    from primus_dlrm_b200.ops.mlp import cross_layer
    torch.manual_seed(d + r)
    U = (torch.randn(d, r, device=DEV) * d ** -0.5).requires_grad_(True)
    V = (torch.randn(r, d, device=DEV) * r ** -0.5).requires_grad_(True)
    b = (0.1 * torch.randn(d, device=DEV)).requires_grad_(True)
    x0 = torch.randn(B, d, device=DEV).to(torch.bfloat16).requires_grad_(True)
    xl = torch.randn(B, d, device=DEV).to(torch.bfloat16).requires_grad_(True)
    y = cross_layer(x0, xl, U, V, b)
    dy = torch.randn(B, d, device=DEV).to(torch.bfloat16)
    y.backward(dy)
    got = [x0.grad.float(), xl.grad.float(), U.grad.clone(), V.grad.clone(), b.grad.clone()]
    for t in (U, V, b):
        t.grad = None
    x0r = x0.detach().float().requires_grad_(True)
    xlr = xl.detach().float().requires_grad_(True)
    yr = x0r * ((xlr @ U) @ V + b) + xlr
    yr.backward(dy.float())
    assert _rel(y, yr) < 2e-2
    ref = [x0r.grad, xlr.grad, U.grad, V.grad, b.grad]
    for name, g, gr in zip(["x0", "xl", "U", "V", "b"], got, ref):
        assert _rel(g, gr) < 3e-2, name


def test_dcnv2_low_rank_module_native_matches_eager():
    """The DCNv2 module (cross layers + deep MLP + combine) on the native path
    against its own eager fp32 forward and backward."""
    from primus_dlrm_b200.models.interaction import DCNv2
    torch.manual_seed(3)
    m = DCNv2(3456, 3, [1024, 1024, 512, 256], dropout=0.0, low_rank=512).to(DEV)
    B = 512
    x = torch.randn(B, 128, device=DEV)
    embs = [torch.randn(B, 128, device=DEV) for _ in range(26)]
    dy = torch.randn(B, 256, device=DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = m(user_features=[x.to(torch.bfloat16)], item_features=[e.to(torch.bfloat16) for e in embs])
    out.float().backward(dy)
    g_native = {n: p.grad.clone() for n, p in m.named_parameters()}
    m.zero_grad()
    out_r = m(user_features=[x], item_features=embs)
    out_r.backward(dy)
    assert _rel(out, out_r) < 3e-2
    # the cross layers and the combining Linear (no ReLU mask between them and
    # the output; the deep MLP's masks are covered by the chain test)
    for n, p in m.named_parameters():
        if n.startswith("cross") or n.startswith("combine"):
            assert _rel(g_native[n], p.grad) < 5e-2, n
