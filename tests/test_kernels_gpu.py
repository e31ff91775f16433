"""sm_100a kernel numerics vs plain-PyTorch fp32 restatements of the same ops."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _tables(rows_list, dim, seed=0):
    from primus_dlrm_b200.ops.embedding import TableShard
    g = torch.Generator(device="cpu").manual_seed(seed)
    out = []
    for i, r in enumerate(rows_list):
        w = (torch.rand(r, dim, generator=g) * 2 - 1).to(DEV)
        out.append(TableShard(name=f"t{i}", rows=r, dim=dim, weight=w))
    return out


def _clone_tables(ts, opt):
    from primus_dlrm_b200.ops.embedding import TableShard
    out = []
    for t in ts:
        c = TableShard(name=t.name, rows=t.rows, dim=t.dim, weight=t.weight.clone())
        c.state = [torch.zeros(s, device=DEV) for s in opt.state_shapes(t.rows, t.dim)]
        out.append(c)
    for t in ts:
        t.state = [torch.zeros(s, device=DEV) for s in opt.state_shapes(t.rows, t.dim)]
    return out


def _spec(tables, slots, shapes, dtype, opt, native):
    from primus_dlrm_b200.ops.embedding import LookupSpec
    return LookupSpec(tables=tables, slots=slots, group_shapes=shapes, dtype=dtype, optimizer=opt,
                      native=native, err=torch.zeros(1, dtype=torch.int32, device=DEV))


@pytest.mark.parametrize("id_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("dim", [16, 64, 128])
def test_gather_grouped(id_dtype, out_dtype, dim):
    from primus_dlrm_b200.ops.embedding import GroupedLookup, Slot, SparseOptimizer
    tables = _tables([1000, 37, 5], dim)
    B, L = 9, 7
    g = torch.Generator().manual_seed(1)
    ids = [torch.randint(0, 1000, (B, L), generator=g), torch.randint(0, 37, (B, L), generator=g),
           torch.randint(0, 5, (B,), generator=g), torch.randint(0, 1000, (B,), generator=g)]
    ids[0][0, :] = 999
    ids[0][1, :] = 0
    ids = [i.to(DEV, id_dtype) for i in ids]
    slots = [Slot(table=0, group=0, col=0), Slot(table=1, group=0, col=dim),
             Slot(table=2, group=1, col=0), Slot(table=0, group=1, col=dim)]
    shapes = [(B, L, 2 * dim), (B, 2 * dim)]
    opt = SparseOptimizer(kind="sgd")
    outs = GroupedLookup.forward(type("C", (), {"save_for_backward": lambda *a: None})(), None,
                                 _spec(tables, slots, shapes, out_dtype, opt, True), *ids)
    ref = [torch.cat([tables[0].weight[ids[0].long()], tables[1].weight[ids[1].long()]], -1),
           torch.cat([tables[2].weight[ids[2].long()], tables[0].weight[ids[3].long()]], -1)]
    for o, r in zip(outs, ref):
        torch.testing.assert_close(o.float(), r.to(out_dtype).float(), rtol=0, atol=0)


@pytest.mark.parametrize("kind", ["sgd", "adagrad", "row_wise_adagrad", "adam"])
@pytest.mark.parametrize("dim", [32, 128])
def test_backward_fused_update(kind, dim):
    from primus_dlrm_b200.ops.embedding import GroupedLookup, Slot, SparseOptimizer
    torch.manual_seed(0)
    rows = [500, 64]
    base = _tables(rows, dim, seed=3)
    opt_n = SparseOptimizer(kind=kind, lr=0.05, eps=1e-6, weight_decay=1e-3)
    opt_e = SparseOptimizer(kind=kind, lr=0.05, eps=1e-6, weight_decay=1e-3)
    ref = _clone_tables(base, opt_n)
    B, L = 33, 50
    ids0 = torch.randint(0, 500, (B, L))
    ids0[:, :20] = 7            # hot row: spans many 32-position chunks
    ids0[0, :] = 499
    ids1 = torch.randint(0, 64, (B, L))
    ids2 = torch.randint(0, 500, (B,))
    ids = [i.to(DEV) for i in (ids0, ids1, ids2)]
    slots = [Slot(table=0, group=0, col=0), Slot(table=1, group=0, col=dim), Slot(table=0, group=1, col=0)]
    shapes = [(B, L, 2 * dim), (B, dim)]
    anchor = torch.zeros((), device=DEV, requires_grad=True)
    for step in range(2):
        grads = [torch.randn(s, device=DEV).to(torch.bfloat16) for s in shapes]
        out_n = GroupedLookup.apply(anchor, _spec(base, slots, shapes, torch.bfloat16, opt_n, True), *ids)
        torch.autograd.backward(out_n, grads)
        out_e = GroupedLookup.apply(anchor, _spec(ref, slots, shapes, torch.bfloat16, opt_e, False), *ids)
        torch.autograd.backward(out_e, grads)
        torch.cuda.synchronize()
        for tn, te in zip(base, ref):
            torch.testing.assert_close(tn.weight, te.weight, rtol=1e-4, atol=1e-5)
            for sn, se in zip(tn.state, te.state):
                torch.testing.assert_close(sn, se, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("pool", [1, 2])
def test_pooled_fwd_bwd(pool):
    from primus_dlrm_b200.ops.embedding import GroupedLookup, Slot, SparseOptimizer
    dim = 64
    base = _tables([300], dim, seed=5)
    opt_n, opt_e = SparseOptimizer(kind="row_wise_adagrad", lr=0.1), SparseOptimizer(kind="row_wise_adagrad", lr=0.1)
    ref = _clone_tables(base, opt_n)
    B, L = 17, 12
    ids = torch.randint(0, 300, (B, L))
    ids[:, -3:] = 0            # padding
    ids[2, :] = 0              # empty bag
    ids = [ids.to(DEV)]
    slots = [Slot(table=0, group=0, col=0, pool=pool, pad_id=0)]
    shapes = [(B, dim)]
    anchor = torch.zeros((), device=DEV, requires_grad=True)
    gr = [torch.randn(B, dim, device=DEV)]
    on = GroupedLookup.apply(anchor, _spec(base, slots, shapes, torch.float32, opt_n, True), *ids)
    oe = GroupedLookup.apply(anchor, _spec(ref, slots, shapes, torch.float32, opt_e, False), *ids)
    torch.testing.assert_close(on[0], oe[0], rtol=1e-5, atol=1e-6)
    torch.autograd.backward(on, gr)
    torch.autograd.backward(oe, gr)
    torch.testing.assert_close(base[0].weight, ref[0].weight, rtol=1e-4, atol=1e-5)


def test_out_of_range_id_sets_error_word():
    from primus_dlrm_b200.ops.embedding import GroupedLookup, Slot, SparseOptimizer
    t = _tables([10], 32)
    spec = _spec(t, [Slot(table=0, group=0, col=0)], [(4, 32)], torch.float32, SparseOptimizer(kind="sgd"), True)
    ids = torch.tensor([1, 2, 10, 3], device=DEV)
    out = GroupedLookup.forward(type("C", (), {"save_for_backward": lambda *a: None})(), None, spec, ids)
    torch.cuda.synchronize()
    assert int(spec.err.item()) == 1
    assert float(out[0][2].abs().sum()) == 0.0


@pytest.mark.parametrize("D", [64, 256, 384, 1024, 2048])
@pytest.mark.parametrize("kind", [0, 1])
def test_norm_fwd_bwd(D, kind):
    from primus_dlrm_b200.ops.norm import _NormFn
    torch.manual_seed(D)
    x = torch.randn(3, 37, D, device=DEV).to(torch.bfloat16).requires_grad_(True)
    w = (torch.rand(D, device=DEV) + 0.5).requires_grad_(True)
    b = torch.randn(D, device=DEV).requires_grad_(True) if kind else None
    y = _NormFn.apply(x, None, w, b, 1e-6, kind)
    xf = x.detach().float().requires_grad_(True)
    wf = w.detach().clone().requires_grad_(True)
    bf = b.detach().clone().requires_grad_(True) if kind else None
    if kind == 0:
        yr = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf
    else:
        yr = torch.nn.functional.layer_norm(xf, (D,), wf, bf, 1e-6)
    torch.testing.assert_close(y.float(), yr, rtol=2e-2, atol=2e-2)
    dy = torch.randn_like(yr)
    y.backward(dy.to(torch.bfloat16))
    yr.backward(dy.to(torch.bfloat16).float())
    torch.testing.assert_close(x.grad.float(), xf.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(w.grad, wf.grad, rtol=2e-2, atol=5e-2)


def test_add_norm_fused():
    from primus_dlrm_b200.ops.norm import add_norm
    a = torch.randn(4, 50, 256, device=DEV).to(torch.bfloat16).requires_grad_(True)
    b = torch.randn(4, 50, 256, device=DEV).to(torch.bfloat16).requires_grad_(True)
    w = torch.ones(256, device=DEV, requires_grad=True)
    y, z = add_norm(a, b, w, None, 1e-6, 0)
    zr = (a.detach().float() + b.detach().float())
    torch.testing.assert_close(z.float(), zr.to(torch.bfloat16).float())
    (y.float().sum() + 2 * z.float().sum()).backward()
    assert a.grad is not None and torch.equal(a.grad, b.grad)


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("D", [256, 384])
def test_add_norm_matches_fp32_reference(kind, D):
    """Fused residual add + norm over a token-sliced (batch-strided) input with
    an odd row count; gradients through both y and z."""
    from primus_dlrm_b200.ops.norm import add_norm
    torch.manual_seed(kind * 7 + D)
    full = torch.randn(3, 45, D, device=DEV).to(torch.bfloat16)
    a = full[:, 6:, :].detach().requires_grad_(True)          # [3, 39, D], batch stride 45 * D
    b = torch.randn(3, 39, D, device=DEV).to(torch.bfloat16).requires_grad_(True)
    w = (torch.rand(D, device=DEV) + 0.5).requires_grad_(True)
    bias = torch.randn(D, device=DEV).requires_grad_(True) if kind else None
    y, z = add_norm(a, b, w, bias, 1e-6, kind)
    af, bf_ = a.detach().float().requires_grad_(True), b.detach().float().requires_grad_(True)
    wf = w.detach().clone().requires_grad_(True)
    biasf = bias.detach().clone().requires_grad_(True) if kind else None
    zf = af + bf_
    if kind == 0:
        yf = zf * torch.rsqrt(zf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf
    else:
        yf = torch.nn.functional.layer_norm(zf, (D,), wf, biasf, 1e-6)
    torch.testing.assert_close(z.float(), zf.to(torch.bfloat16).float())
    torch.testing.assert_close(y.float(), yf, rtol=2e-2, atol=3e-2)
    gy = torch.randn_like(yf).to(torch.bfloat16)
    gz = torch.randn_like(zf).to(torch.bfloat16)
    torch.autograd.backward([y, z], [gy, gz])
    torch.autograd.backward([yf, zf], [gy.float(), gz.float()])
    torch.testing.assert_close(a.grad.float(), af.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(b.grad.float(), bf_.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(w.grad, wf.grad, rtol=2e-2, atol=1e-1)
    if kind:
        torch.testing.assert_close(bias.grad, biasf.grad, rtol=2e-2, atol=1e-1)


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("q_len", [40, 17, 5])
def test_norm_with_tail_gradient(kind, q_len):
    """(norm(x), x[:, T-q:]) in one node: the tail's gradient is added inside
    the norm backward; compared with the fp32 autograd of the same graph."""
    from primus_dlrm_b200.ops.norm import make_norm, norm_with_tail
    torch.manual_seed(q_len + kind)
    D, T = 256, 40
    norm = make_norm("rmsnorm" if kind == 0 else "layernorm", D).to(DEV)
    with torch.no_grad():
        norm.weight.uniform_(0.5, 1.5)
        if kind:
            norm.bias.normal_()
    x = torch.randn(3, T, D, device=DEV).to(torch.bfloat16).requires_grad_(True)
    y, tail = norm_with_tail(norm, x, q_len)
    assert tail.shape == (3, q_len, D) and torch.equal(tail, x[:, T - q_len:])
    gy = torch.randn(3, T, D, device=DEV).to(torch.bfloat16)
    gt = torch.randn(3, q_len, D, device=DEV).to(torch.bfloat16)
    torch.autograd.backward([y, tail * 1.0], [gy, gt])
    xf = x.detach().float().requires_grad_(True)
    wf = norm.weight.detach().clone().requires_grad_(True)
    if kind == 0:
        yf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + norm.eps) * wf
    else:
        yf = torch.nn.functional.layer_norm(xf, (D,), wf, norm.bias.detach(), norm.eps)
    torch.autograd.backward([yf, xf[:, T - q_len:]], [gy.float(), gt.float()])
    torch.testing.assert_close(y.float(), yf, rtol=2e-2, atol=3e-2)
    torch.testing.assert_close(x.grad.float(), xf.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(norm.weight.grad, wf.grad, rtol=2e-2, atol=1e-1)


def test_heads_loss():
    from primus_dlrm_b200.ops.loss import _HeadsLossFn, heads_loss_ref
    torch.manual_seed(0)
    B, D, T = 1000, 96, 3
    h = torch.randn(B, D, device=DEV).to(torch.bfloat16).requires_grad_(True)
    W = (torch.randn(T, D, device=DEV) * 0.1).requires_grad_(True)
    b = torch.randn(T, device=DEV).requires_grad_(True)
    y = torch.stack([(torch.rand(B, device=DEV) < 0.3).float(), (torch.rand(B, device=DEV) < 0.1).float(),
                     torch.rand(B, device=DEV)])
    tw, reg = [1.0, 0.5, 2.0], [0, 0, 1]
    tot, per, lg = _HeadsLossFn.apply(h, W, b, y, tw, reg)
    hr, Wr, br = h.detach().float().requires_grad_(True), W.detach().clone().requires_grad_(True), \
        b.detach().clone().requires_grad_(True)
    tr, pr, lr = heads_loss_ref(hr, Wr, br, y, tw, reg)
    torch.testing.assert_close(tot, tr, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(per, pr, rtol=1e-4, atol=1e-5)
    (2.0 * tot).backward()
    (2.0 * tr).backward()
    torch.testing.assert_close(h.grad.float(), hr.grad, rtol=2e-2, atol=1e-4)
    torch.testing.assert_close(W.grad, Wr.grad, rtol=1e-3, atol=1e-5)
    torch.testing.assert_close(b.grad, br.grad, rtol=1e-3, atol=1e-5)


def test_fused_adamw_matches_torch():
    from primus_dlrm_b200.ops.optim import FlatParams, FusedAdamW
    torch.manual_seed(0)
    ps = [torch.nn.Parameter(torch.randn(s, device=DEV)) for s in [(33, 7), (129,), (5, 5, 5)]]
    ref = [torch.nn.Parameter(p.detach().clone()) for p in ps]
    flat = FlatParams(ps)
    opt = FusedAdamW(flat, lr=1e-2, weight_decay=0.1, max_grad_norm=0.5)
    topt = torch.optim.AdamW(ref, lr=1e-2, weight_decay=0.1)
    for _ in range(3):
        flat.zero_grad()
        grads = [torch.randn_like(p) for p in ps]
        for p, r, g in zip(ps, ref, grads):
            p.grad.copy_(g)
            r.grad = g.clone()
        torch.nn.utils.clip_grad_norm_(ref, 0.5)
        opt.step()
        topt.step()
    for p, r in zip(ps, ref):
        torch.testing.assert_close(p.detach(), r.detach(), rtol=1e-5, atol=1e-6)


def test_onetrans_native_matches_eager_one_step():
    """Tiny OneTrans: native kernels vs eager PyTorch, same weights and batch."""
    import copy
    import os

    from primus_dlrm_b200.config import Config
    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.models.onetrans import OneTransModel
    cfg = Config.load(os.path.join(os.path.dirname(__file__), "..", "configs", "onetrans_tiny.yaml"))
    torch.manual_seed(0)
    m_native = OneTransModel(cfg, device=DEV)
    m_eager = copy.deepcopy(m_native)
    m_eager.emb.native = False
    for m in (m_native, m_eager):
        for t in m.emb.tables():
            t.shard.weight = t.weight.data
    batch = {k: v.to(DEV) for k, v in generate_batch(cfg, 32, seed=3).items()}
    with torch.autocast("cuda", dtype=torch.bfloat16):
        tn, _, _ = m_native.forward_loss(batch, cfg.train.loss_weights, cfg.train.regression_tasks)
    os.environ["PD_KERNELS"] = "eager"
    try:
        with torch.autocast("cuda", dtype=torch.bfloat16):
            te, _, _ = m_eager.forward_loss(batch, cfg.train.loss_weights, cfg.train.regression_tasks)
    finally:
        os.environ.pop("PD_KERNELS")
    assert math.isfinite(tn.item())
    torch.testing.assert_close(tn.float(), te.float(), rtol=3e-2, atol=3e-2)
