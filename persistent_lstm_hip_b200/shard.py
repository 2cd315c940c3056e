"""Batch sharding of the LSTM + Linear forward over several GPUs.

Batch rows are independent sequences, so the forward shards by rows with no
collective on the hot path: every device runs the whole stack on its rows with
replicated weights, and the only cross-device traffic is the final output
gather.  The reference is single-device (every kernel on one stream of one
device, persistent_lstm_hip.cu:1967-1972); this module adds the partition.

* ``plan_shards``: contiguous row ranges for uniform lengths; for variable
  lengths the rows are sorted by length (longest first) and dealt round-robin,
  so every shard gets the same row count and nearly the same total and maximum
  length (balanced kernel time).
* ``MultiDeviceRegressor``: one process driving N devices (one stream each);
  inputs are scattered and outputs gathered with peer copies over NVLink.
* ``distributed_forward``: one process per GPU (torchrun); each rank runs its
  shard, then a single all-gather (NCCL on GPUs, gloo on CPU) assembles the
  batch in original row order on every rank.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch


def plan_shards(batch: int, n_shards: int, lengths: Optional[Sequence[int]] = None) -> List[torch.Tensor]:
    """Row indices (int64, CPU) of each shard; their concatenation is a permutation of range(batch)."""
    if n_shards < 1:
        raise ValueError("n_shards must be >= 1")
    if lengths is None:
        bounds = [batch * i // n_shards for i in range(n_shards + 1)]
        return [torch.arange(bounds[i], bounds[i + 1], dtype=torch.int64) for i in range(n_shards)]
    lens = torch.as_tensor(lengths, dtype=torch.int64).cpu()
    if lens.numel() != batch:
        raise ValueError(f"lengths has {lens.numel()} entries, expected {batch}")
    order = torch.sort(lens, descending=True, stable=True).indices
    return [order[i::n_shards].clone() for i in range(n_shards)]


def shard_balance(plan: Sequence[torch.Tensor], lengths: Optional[Sequence[int]] = None) -> dict:
    """Rows, total length and maximum length of every shard (a load-balance report)."""
    lens = None if lengths is None else torch.as_tensor(lengths, dtype=torch.int64).cpu()
    rep = []
    for idx in plan:
        if lens is None:
            rep.append({"rows": int(idx.numel())})
        else:
            sel = lens[idx]
            rep.append({"rows": int(idx.numel()), "sum_len": int(sel.sum()) if sel.numel() else 0,
                        "max_len": int(sel.max()) if sel.numel() else 0})
    return {"shards": rep}


def _unpermute(parts: Sequence[torch.Tensor], plan: Sequence[torch.Tensor], batch: int, dim: int = 0) -> torch.Tensor:
    cat = torch.cat(list(parts), dim=dim)
    perm = torch.cat(list(plan)).to(cat.device)
    out = torch.empty_like(cat)
    out.index_copy_(dim, perm, cat)
    assert out.shape[dim] == batch
    return out


class MultiDeviceRegressor:
    """One process, N devices: the forward of a PersistentLSTMRegressor sharded by rows.

    `model` is replicated to every device in `devices` (weights are small); each
    call scatters x (and lengths) by `plan_shards`, launches every shard on its
    device's current stream, and gathers [B, O] (or [B, T, O] for
    forward_sequence) onto devices[0] in the original row order.
    """

    def __init__(self, model, devices: Sequence[torch.device]):
        import copy

        if len(devices) < 1:
            raise ValueError("at least one device is required")
        self.devices = [torch.device(d) for d in devices]
        self.replicas = []
        for d in self.devices:
            rep = copy.deepcopy(model).to(d)
            self.replicas.append(rep)

    def _run(self, x: torch.Tensor, lengths, seq: bool):
        B = int(x.shape[0])
        lens_cpu = None if lengths is None else torch.as_tensor(lengths).cpu()
        plan = plan_shards(B, len(self.devices), None if lens_cpu is None else lens_cpu.tolist())
        outs, states = [], []
        for dev, rep, idx in zip(self.devices, self.replicas, plan):
            with torch.cuda.device(dev):
                xs = x.index_select(0, idx.to(x.device)).to(dev, non_blocking=True)
                ls = None if lens_cpu is None else lens_cpu[idx].to(dev, non_blocking=True)
                if seq:
                    o, (h, c) = rep.forward_sequence(xs, lengths=ls)
                    states.append((h, c))
                else:
                    o = rep(xs, lengths=ls)
                outs.append(o)
        home = self.devices[0]
        gathered = [o.to(home, non_blocking=True) for o in outs]
        out = _unpermute(gathered, plan, B, dim=0)
        if not seq:
            return out
        h = _unpermute([s[0].to(home, non_blocking=True) for s in states], plan, B, dim=1)
        c = _unpermute([s[1].to(home, non_blocking=True) for s in states], plan, B, dim=1)
        return out, (h, c)

    def __call__(self, x: torch.Tensor, lengths=None) -> torch.Tensor:
        return self._run(x, lengths, seq=False)

    def forward_sequence(self, x: torch.Tensor, lengths=None):
        return self._run(x, lengths, seq=True)


def distributed_forward(fn: Callable[[torch.Tensor, Optional[torch.Tensor]], torch.Tensor],
                        x_local: torch.Tensor, plan: Sequence[torch.Tensor],
                        lengths_local: Optional[torch.Tensor] = None, group=None) -> torch.Tensor:
    """Runs `fn(x_local, lengths_local)` on this rank's rows and all-gathers the results.

    `plan` is the same list of row-index shards on every rank (plan_shards over
    the global batch, one shard per rank, equal row counts); `x_local` holds
    the rows plan[rank].  Returns the [B, ...] output in original row order on
    every rank.  The all-gather is the path's only collective.
    """
    import torch.distributed as dist

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    if len(plan) != world:
        raise ValueError(f"plan has {len(plan)} shards for {world} ranks")
    if int(x_local.shape[0]) != int(plan[rank].numel()):
        raise ValueError("x_local rows do not match this rank's shard")
    out_local = fn(x_local, lengths_local).contiguous()
    parts = [torch.empty_like(out_local) for _ in range(world)]
    dist.all_gather(parts, out_local, group=group)
    return _unpermute(parts, plan, sum(int(p.numel()) for p in plan), dim=0)
