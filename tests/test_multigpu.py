"""Multi-GPU (every visible GPU up to 8, at least 2; NCCL): the NVLink
peer-memory sparse exchange against the collective baseline, the dense peer
collectives against NCCL, the bucketed gradient sync overlapped with the
backward against the sync after it, and a bounded barrier.  Needs 2+ CUDA
devices."""
import os

import pytest
import torch

from dist_utils import free_port

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = os.path.join(ROOT, "configs", "onetrans_tiny.yaml")


def _nccl_entry(rank, world, port, fn, q):
    import datetime
    import traceback

    import torch.distributed as dist
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank), "NCCL_NVLS_ENABLE": "0"})
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        out = fn(rank, world)
        import io
        buf = io.BytesIO()
        torch.save(out, buf)
        q.put((rank, "ok", buf.getvalue()))
    except BaseException:
        q.put((rank, "err", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_nccl(fn, world=2):
    import io

    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_nccl_entry, args=(r, world, port, fn, q)) for r in range(world)]
    for p in ps:
        p.start()
    res, errs = {}, []
    for _ in range(world):
        r, st, v = q.get(timeout=600)
        if st == "ok":
            res[r] = torch.load(io.BytesIO(v), weights_only=False)
        else:
            errs.append(v)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    if errs:
        raise RuntimeError("\n".join(errs))
    return res


def _world() -> int:
    return min(torch.cuda.device_count(), 8)


def _cfg(comm, opt="sgd"):
    from primus_dlrm_b200.config import Config, TableShardingSpec
    cfg = Config.load(TINY)
    kinds = {"item": "row_wise", "artist": "table_wise", "album": "column_wise", "uid": "data_parallel"}
    for t in cfg.model.embedding_tables:
        t.sharding = TableShardingSpec(sharding_type=kinds[t.name], ranks=[1] if t.name == "artist" else None)
    cfg.distributed.embedding_sharding.enabled = True
    cfg.distributed.comm = comm
    cfg.train.embedding_optimizer = opt
    cfg.train.bf16 = False
    cfg.train.warmup_steps = 1
    return cfg


def _peer_vs_nccl(rank, world):
    import copy

    import torch.distributed as dist

    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.parallel.build import build_model
    from primus_dlrm_b200.parallel.state import full_state_dict, load_full_state_dict
    from primus_dlrm_b200.parallel.wrapper import wrap_model
    from primus_dlrm_b200.training.engine import TrainEngine
    dev = torch.device("cuda", rank)
    out = {}
    torch.manual_seed(0)
    init = copy.deepcopy(build_model(_cfg("nccl")).state_dict())
    for comm in ("peer", "nccl"):
        cfg = _cfg(comm)
        model = build_model(cfg, device=dev, meta_device=True)
        model, sync = wrap_model(model, dev, cfg)
        load_full_state_dict(model, init)
        eng = TrainEngine(model, cfg, dev, grad_sync=sync)
        losses = []
        for s in range(3):
            b = generate_batch(cfg, 32, seed=1000 * s + rank)
            loss, _ = eng.step({k: v.to(dev) for k, v in b.items()})
            losses.append(float(loss))
        ex = model.emb.executor
        if hasattr(ex, "check"):
            ex.check()
        model.emb.check_errors()
        out[comm] = (losses, full_state_dict(model))
        dist.barrier()
    return out


def test_peer_exchange_matches_collective_baseline():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_nccl(_peer_vs_nccl, _world())
    for r in range(_world()):
        lp, ln = res[r]["peer"][0], res[r]["nccl"][0]
        assert lp == pytest.approx(ln, rel=2e-3, abs=2e-3)
    sd_p, sd_n = res[0]["peer"][1], res[0]["nccl"][1]
    for k in sd_n:
        torch.testing.assert_close(sd_p[k], sd_n[k], rtol=2e-3, atol=2e-4, msg=lambda m: f"{k}: {m}")


def _barrier_timeout(rank, world):
    """A barrier whose peer never arrives returns an error status (no hang)."""
    from primus_dlrm_b200.ops import _ext
    from primus_dlrm_b200.parallel.sharded_embedding import SymmetricBuffer
    dev = torch.device("cuda", rank)
    pads = SymmetricBuffer(64 * 8, dev, rank, world)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ptrs = torch.tensor(pads.ptrs, dtype=torch.int64)
    if rank == 0:  # only rank 0 enters: its wait for rank 1 must time out
        _ext.core().signal_barrier(ptrs, rank, 5, int(0.5e9), err)
    torch.cuda.synchronize()
    import torch.distributed as dist
    dist.barrier()
    return int(err.item())


def test_barrier_wait_is_bounded():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_nccl(_barrier_timeout, 2)
    assert res[0] == 2 and res[1] == 0


def _dense_peer_collectives(rank, world):
    """Peer-memory DDP all-reduce and ZeRO reduce-scatter / all-gather vs NCCL."""
    import torch.distributed as dist

    from primus_dlrm_b200.parallel.wrapper import PeerGradSync, PeerShardedGradSync
    dev = torch.device("cuda", rank)
    n = 1_000_003 * 4 + 36            # not a multiple of the slice alignment
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(n, device=dev, generator=g)
    ref = x.clone()
    dist.all_reduce(ref)
    ref /= world

    class _Flat:                        # the FlatParams surface the syncs use
        def __init__(self, n):
            self.numel = n
            self.grad = torch.zeros(n, device=dev)
            self.data = torch.zeros(n, device=dev)

        def zero_grad(self):
            pass

        def rebind_all(self):
            pass

    f = _Flat(n)
    s = PeerGradSync(n, dev)
    s.bind(f)
    out = {}
    for it in range(3):                 # repeated use: barriers / epochs advance
        f.grad.copy_(x * (it + 1))
        s.sync(f.grad)
        torch.cuda.synchronize()
        s.check()
        out[f"ddp{it}"] = (f.grad - ref * (it + 1)).abs().max().item()
    z = PeerShardedGradSync(n, dev)
    fz = _Flat(n)
    z.bind(fz)
    fz.grad.copy_(x)
    z.sync(fz.grad)
    a, b = z.shard_range(n)
    out["rs"] = (fz.grad[a:b] - ref[a:b]).abs().max().item()
    fz.data.copy_(x)                     # each rank's own slice is authoritative
    z.gather_params(fz.data)
    full = [torch.empty(n, device=dev) for _ in range(world)]
    dist.all_gather(full, x)
    expect = torch.empty(n, device=dev)
    for r in range(world):
        lo, hi = z.bounds[r].item(), z.bounds[r + 1].item()
        expect[lo:hi] = full[r][lo:hi]
    torch.cuda.synchronize()
    z.check()
    out["ag"] = (fz.data - expect).abs().max().item()
    return out


def test_dense_peer_collectives_match_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_nccl(_dense_peer_collectives, _world())
    for r, d in res.items():
        for k, v in d.items():
            assert v < 1e-5, (r, k, v)


def _overlap_vs_sync(rank, world):
    """The same steps with the bucketed gradient sync overlapped with the
    backward (many small buckets) and with one all-reduce after it."""
    import copy

    import torch.distributed as dist

    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.parallel.build import build_model
    from primus_dlrm_b200.parallel.state import full_state_dict, load_full_state_dict
    from primus_dlrm_b200.parallel.wrapper import wrap_model
    from primus_dlrm_b200.training.engine import TrainEngine
    dev = torch.device("cuda", rank)
    torch.manual_seed(0)
    init = copy.deepcopy(build_model(_cfg("peer")).state_dict())
    out = {}
    for mode in ("1", "0"):
        os.environ["PD_OVERLAP_DENSE_SYNC"] = mode
        os.environ["PD_DDP_BUCKET_MB"] = "0.05"        # tens of buckets on the tiny model
        cfg = _cfg("peer")
        model = build_model(cfg, device=dev, meta_device=True)
        model, sync = wrap_model(model, dev, cfg)
        load_full_state_dict(model, init)
        eng = TrainEngine(model, cfg, dev, grad_sync=sync)
        if mode == "1":
            out["buckets"] = len(sync.impl.buckets)
        losses = []
        for s in range(3):
            b = generate_batch(cfg, 32, seed=1000 * s + rank)
            loss, _ = eng.step({k: v.to(dev) for k, v in b.items()})
            losses.append(float(loss))
        torch.cuda.synchronize()
        sync.impl.check()
        sd = full_state_dict(model)
        out[mode] = (losses, {k: v for k, v in sd.items() if not k.startswith("emb.")})
        dist.barrier()
    os.environ.pop("PD_OVERLAP_DENSE_SYNC", None)
    os.environ.pop("PD_DDP_BUCKET_MB", None)
    return out


def test_overlapped_bucket_sync_matches_sync_after_backward():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_nccl(_overlap_vs_sync, _world())
    assert res[0]["buckets"] > 4
    # not bitwise: the sparse exchange's atomics already perturb the first
    # loss (before any gradient sync) in the last bits between two runs
    for r, d in res.items():
        assert d["1"][0] == pytest.approx(d["0"][0], rel=1e-4, abs=1e-5), (r, d["1"][0], d["0"][0])
    sd1, sd0 = res[0]["1"][1], res[0]["0"][1]
    for k in sd0:
        torch.testing.assert_close(sd1[k], sd0[k], rtol=1e-3, atol=1e-5, msg=lambda m: f"{k}: {m}")


def _fsdp_vs_ddp(rank, world):
    """The same bf16 steps with FSDP-sharded dense parameters and with the
    replicated (DDP) arena: losses agree to bf16 rounding and each FSDP rank
    holds 1/W of the dense parameters."""
    import copy

    import torch.distributed as dist

    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.parallel.build import build_model
    from primus_dlrm_b200.parallel.fsdp import DTensor
    from primus_dlrm_b200.parallel.state import full_state_dict, load_full_state_dict
    from primus_dlrm_b200.parallel.wrapper import wrap_model
    from primus_dlrm_b200.training.engine import TrainEngine
    dev = torch.device("cuda", rank)
    torch.manual_seed(0)

    def cfg_of(dense):
        cfg = _cfg("peer", opt="adam")
        cfg.model.transformer.d_model = 128
        cfg.distributed.dense_strategy = dense
        cfg.train.bf16 = True
        return cfg
    init = copy.deepcopy(build_model(cfg_of("ddp")).state_dict())
    out = {}
    for dense in ("fsdp", "ddp"):
        cfg = cfg_of(dense)
        model = build_model(cfg, device=dev, meta_device=True)
        model, sync = wrap_model(model, dev, cfg)
        load_full_state_dict(model, init)
        eng = TrainEngine(model, cfg, dev, grad_sync=sync)
        losses = []
        for s in range(4):
            b = generate_batch(cfg, 64, seed=1000 * s + rank)
            loss, _ = eng.step({k: v.to(dev) for k, v in b.items()})
            losses.append(float(loss))
        torch.cuda.synchronize()
        ps = [p for n, p in model.named_parameters() if p.requires_grad and not n.startswith("emb")]
        local = sum((p.to_local() if isinstance(p, DTensor) else p).numel() for p in ps)
        sd = full_state_dict(model)
        out[dense] = (losses, local, sum(p.numel() for p in ps),
                      {k: v for k, v in sd.items() if not k.startswith("emb.")})
        dist.barrier()
        del eng, model
    return out


def test_fsdp_matches_ddp_and_shards_parameters():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = _world()
    res = run_nccl(_fsdp_vs_ddp, world)
    for r, d in res.items():
        lf, ld = d["fsdp"][0], d["ddp"][0]
        assert lf == pytest.approx(ld, rel=2e-2, abs=2e-2), (r, lf, ld)
        local, full = d["fsdp"][1], d["fsdp"][2]
        assert local < full / world * 1.1 + 4096, (local, full)
        assert d["ddp"][1] == full
    sf, sd = res[0]["fsdp"][3], res[0]["ddp"][3]
    assert set(sf) == set(sd)
    # Adam moves every weight by about lr per step whatever the gradient's
    # size, so a bf16 rounding flip of a tiny gradient's sign can move a weight
    # by up to 2 lr per step: 4 steps at lr 1e-3
    for k in sd:
        torch.testing.assert_close(sf[k].float(), sd[k].float(), rtol=0, atol=8e-3, msg=lambda m: f"{k}: {m}")


def _pooled_cfg(comm):
    from primus_dlrm_b200.config import Config, TableShardingSpec
    cfg = Config.load(os.path.join(os.path.dirname(TINY), "dlrm_baseline.yaml"))
    cfg.data.history_length = 12
    cfg.model.dropout = 0.0
    kinds = {"hist_item": "row_wise", "item": "row_wise", "hist_artist": "table_wise", "artist": "table_wise",
             "hist_album": "row_wise", "album": "data_parallel", "uid": "row_wise"}
    for t in cfg.model.embedding_tables:
        t.num_embeddings = {"hist_item": 5003, "item": 5003, "hist_artist": 701, "artist": 701,
                            "hist_album": 1301, "album": 1301, "uid": 997}[t.name]
        t.sharding = TableShardingSpec(sharding_type=kinds[t.name], ranks=[1] if "artist" in t.name else None)
    cfg.distributed.embedding_sharding.enabled = True
    cfg.distributed.comm = comm
    cfg.train.embedding_optimizer = "row_wise_adagrad"
    cfg.train.bf16 = False
    cfg.train.warmup_steps = 1
    return cfg


def _pooled_peer_vs_nccl(rank, world):
    """DLRM two-tower (mean-pooled history bags) with the peer-memory exchange
    against the NCCL all-to-all baseline: same losses and tables."""
    import copy

    import torch.distributed as dist

    from primus_dlrm_b200.data.synthetic import generate_batch
    from primus_dlrm_b200.parallel.build import build_model
    from primus_dlrm_b200.parallel.state import full_state_dict, load_full_state_dict
    from primus_dlrm_b200.parallel.wrapper import wrap_model
    from primus_dlrm_b200.training.engine import TrainEngine
    dev = torch.device("cuda", rank) if torch.cuda.is_available() else torch.device("cpu")
    torch.manual_seed(0)
    init = copy.deepcopy(build_model(_pooled_cfg("nccl")).state_dict())
    out = {}
    for comm in (("peer", "nccl") if dev.type == "cuda" else ("nccl",)):
        cfg = _pooled_cfg(comm)
        model = build_model(cfg, device=dev, meta_device=True)
        model, sync = wrap_model(model, dev, cfg)
        load_full_state_dict(model, init)
        eng = TrainEngine(model, cfg, dev, grad_sync=sync)
        assert any(model.emb.is_pooled(f) for f in cfg.feature.all_ec_feature_names())
        losses = []
        for s in range(3):
            b = generate_batch(cfg, 64, seed=1000 * s + rank)
            loss, _ = eng.step({k: v.to(dev) for k, v in b.items()})
            losses.append(float(loss))
        model.emb.check_errors()
        out[comm] = (losses, full_state_dict(model))
        dist.barrier()
    return out


def test_pooled_peer_exchange_matches_collective_baseline():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = run_nccl(_pooled_peer_vs_nccl, min(_world(), 2))
    for r in res:
        assert res[r]["peer"][0] == pytest.approx(res[r]["nccl"][0], rel=2e-3, abs=2e-3)
    sd_p, sd_n = res[0]["peer"][1], res[0]["nccl"][1]
    for k in sd_n:
        torch.testing.assert_close(sd_p[k], sd_n[k], rtol=2e-3, atol=2e-4, msg=lambda m: f"{k}: {m}")
