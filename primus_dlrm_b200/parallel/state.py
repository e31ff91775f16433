"""Full (unsharded) state dicts of a sharded model.

``full_state_dict`` assembles every embedding table (and, optionally, its
sparse-optimizer state) on ``dst`` from the shards of all ranks; dense
parameters are identical on every rank and come from ``dst``'s copy.  The
key layout is the reference's (``emb.ec.embeddings.<t>.weight`` ...), so
the result is a plain single-process state dict
(``primus_dlrm/training/dist_trainer.py:39-63`` gathers DMP shards with a
``dist.reduce`` of zero-padded full tables; here row blocks are gathered
with ``dist.gather`` in bounded chunks, so no rank ever holds W copies).
FSDP-sharded dense parameters are gathered with ``DTensor.full_tensor``.

``load_full_state_dict`` slices a full state dict into this rank's shards.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from primus_dlrm_b200.parallel.fsdp import DTensor, full_tensor, local_chunk

_CHUNK_ROWS = 1 << 20


def _is_table_key(model, key: str):
    inner = getattr(model, "module", model)
    emb = getattr(inner, "emb", None)
    if emb is None:
        return None
    for t in emb.tables():
        if key.endswith(f".{t.name}.weight") and (".embeddings." in key or ".embedding_bags." in key):
            return t
    return None


def _gather_rows(local: torch.Tensor, rows_of: list[int], dst: int, rank: int, world: int, group) -> torch.Tensor | None:
    """Concatenate the row blocks ``local`` of all ranks on ``dst`` (CPU result)."""
    shape_tail = tuple(local.shape[1:])
    out = torch.empty((sum(rows_of),) + shape_tail, dtype=local.dtype) if rank == dst else None
    mx = max(rows_of) if rows_of else 0
    offsets = [sum(rows_of[:r]) for r in range(world)]
    for s in range(0, mx, _CHUNK_ROWS):
        e = min(s + _CHUNK_ROWS, mx)
        piece = torch.zeros((e - s,) + shape_tail, dtype=local.dtype, device=local.device)
        n_mine = max(min(local.shape[0], e) - s, 0)
        if n_mine > 0:
            piece[:n_mine] = local[s:s + n_mine]
        bufs = [torch.empty_like(piece) for _ in range(world)] if rank == dst else None
        dist.gather(piece, bufs, dst=dst, group=group)
        if rank == dst:
            for r in range(world):
                n_r = max(min(rows_of[r], e) - s, 0)
                if n_r:
                    out[offsets[r] + s: offsets[r] + s + n_r] = bufs[r][:n_r].cpu()
    return out


def _full_table(t, tensor: torch.Tensor, dst: int, rank: int, world: int, group):
    plan = getattr(t, "plan", None)
    kind = plan.kind if plan is not None else "data_parallel"
    if kind == "row_wise":
        rows_of = [0] * world
        n = torch.tensor([tensor.shape[0]], device=tensor.device)
        ns = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(ns, n, group=group)
        rows_of = [int(x) for x in ns]
        return _gather_rows(tensor, rows_of, dst, rank, world, group)
    if kind == "column_wise":
        # rank q holds all rows of column block q; 1-D states (row-wise
        # accumulators) are kept per block and gather as [rows, W]
        x = tensor if tensor.dim() == 2 else tensor[:, None]
        rows = x.shape[0]
        blocks = []
        for q in range(world):
            local = x if rank == q else x[:0]
            blocks.append(_gather_rows(local, [rows if r == q else 0 for r in range(world)], dst, rank, world, group))
        return torch.cat(blocks, dim=1) if rank == dst else None
    if kind == "table_wise":
        rows_of = [t.num_embeddings if r == plan.owner else 0 for r in range(world)]
        return _gather_rows(tensor, rows_of, dst, rank, world, group)
    return tensor.detach().cpu() if rank == dst else None


def full_state_dict(model, dst: int = 0, group=None, with_optimizer_state: bool = False) -> dict:
    """Single-process state dict on ``dst`` ({} on other ranks).  With
    ``with_optimizer_state`` the sparse optimizer state is returned too, under
    ``"__sparse_state__"``: {table: [state tensors]}."""
    inner = getattr(model, "module", model)
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        sd = {k: v.detach().cpu() for k, v in inner.state_dict().items()}
        if with_optimizer_state and hasattr(inner, "emb"):
            sd["__sparse_state__"] = {t.name: [s.cpu() for s in t.opt_state] for t in inner.emb.tables()}
        return sd
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    out = {}
    for k, v in inner.state_dict().items():
        t = _is_table_key(model, k)
        if t is None:
            v = full_tensor(v.detach())              # FSDP shards: gathered on every rank
            if rank == dst:
                out[k] = v.cpu()
            continue
        full = _full_table(t, v.detach(), dst, rank, world, group)
        if rank == dst:
            out[k] = full
    if with_optimizer_state and hasattr(inner, "emb"):
        st = {}
        for t in inner.emb.tables():
            t.ensure_state(inner.emb.optimizer)
            st[t.name] = [_full_table(t, s, dst, rank, world, group) for s in t.opt_state]
        if rank == dst:
            out["__sparse_state__"] = st
    return out if rank == dst else {}


def _local_slice(t, full: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    plan = getattr(t, "plan", None)
    kind = plan.kind if plan is not None else "data_parallel"
    if kind == "row_wise":
        a = t.shard.local_row0
        return full[a:a + t.shard.local_rows]
    if kind == "column_wise":
        if full.dim() == 2 and full.shape[1] == world and t.weight.shape[1] != world:
            return full[:, rank]          # per-block 1-D state gathered as [rows, W]
        c = t.weight.shape[1]
        return full[:, rank * c:(rank + 1) * c]
    if kind == "table_wise":
        return full if plan.owner == rank else full[:0]
    return full


def load_full_state_dict(model, sd: dict, strict: bool = True) -> None:
    """Load a single-process state dict into a (possibly sharded) model."""
    inner = getattr(model, "module", model)
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    sd = {_canonical(k): v for k, v in sd.items() if k != "__sparse_state__"}
    own = inner.state_dict()
    missing = [k for k in own if k not in sd]
    unexpected = [k for k in sd if k not in own]
    if strict and (missing or unexpected):
        raise KeyError(f"state dict mismatch: missing={missing[:8]} unexpected={unexpected[:8]}")
    with torch.no_grad():
        for k, v in own.items():
            if k not in sd:
                continue
            t = _is_table_key(model, k)
            src = sd[k]
            if t is not None:
                src = _local_slice(t, src, rank, world)
            if isinstance(v, DTensor):                # an FSDP shard: this rank's dim-0 chunk
                v.to_local().copy_(local_chunk(src, v).to(v.dtype))
                continue
            v.copy_(src.to(v.dtype))
    if hasattr(inner, "emb"):
        for t in inner.emb.tables():
            t.shard.weight = t.weight.data


def load_sparse_state(model, st: dict) -> None:
    inner = getattr(model, "module", model)
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    for t in inner.emb.tables():
        if t.name not in st:
            continue
        t.ensure_state(inner.emb.optimizer)
        for dst, src in zip(t.opt_state, st[t.name]):
            dst.copy_(_local_slice(t, src, rank, world).to(dst.device))


def _canonical(key: str) -> str:
    """Strip wrapper prefixes (``_orig_mod.`` of torch.compile, ``module.``)."""
    return key.replace("._orig_mod.", ".").replace("_orig_mod.", "").removeprefix("module.")
