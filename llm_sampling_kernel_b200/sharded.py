"""Multi-GPU use of the fused sampler: one process per GPU, torch.distributed for the plumbing.

Two layouts, the two ways the path shards:

* **Batch-sharded rows** (:class:`BatchShardedSampler`): rank r owns rows
  ``[r*B/w, (r+1)*B/w)``. Rows are independent, so there is no collective on the data path; the
  per-row uniform is evaluated at the global row index (``row_base``), so a sharded run draws
  exactly what a single-GPU run over the whole batch draws. An all-gather of the B int64 ids is
  offered for callers that need every id on every rank.
* **Vocab-sharded tensor parallelism** (:class:`VocabShardedSampler`): rank r holds the
  contiguous logit columns ``[r*V/w, (r+1)*V/w)`` of every row. Each rank selects its local top-k
  as packed (order key, global id) words -- ids offset by the shard base so the lowest-id tie
  rule stays exact across shards -- the K+1 words per row (K candidates + the shard's row status)
  are all-gathered, and every rank merges the w*K candidates and samples with the same uniform,
  so all ranks emit identical ids. The exchange is B*(K+1)*8 bytes per rank.

Both take an ``ops`` object (default: the CUDA operator module) so the host logic can be driven
by another implementation of the same four calls.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) of n items for `rank` of `world`; the first n % world ranks get one more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def _default_ops():
    from . import ops

    return ops()


@dataclass
class BatchShardedSampler:
    """Samples this rank's rows of a batch-sharded [B, V] logits matrix."""

    batch: int
    group: Optional[dist.ProcessGroup] = None
    ops: object = None

    def __post_init__(self):
        self.world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        self.rows = shard_range(self.batch, self.world, self.rank)
        if self.ops is None:
            self.ops = _default_ops()

    def sample(self, local_logits: torch.Tensor, top_k: int, top_p: float, *, seed: int, offset: int,
               uniforms: Optional[torch.Tensor] = None, gather: bool = False) -> torch.Tensor:
        lo, hi = self.rows
        if local_logits.shape[0] != hi - lo:
            raise ValueError(f"rank {self.rank} holds rows [{lo}, {hi}) but got {local_logits.shape[0]}")
        ids = self.ops.sample_ex(local_logits, top_k, top_p, None, None, uniforms, seed, offset, 0, 0, lo,
                                 False)[0]
        if not gather or self.world == 1:
            return ids
        sizes = [shard_range(self.batch, self.world, r) for r in range(self.world)]
        bufs = [torch.empty(h - l, dtype=ids.dtype, device=ids.device) for l, h in sizes]
        dist.all_gather(bufs, ids, group=self.group)
        return torch.cat(bufs)


@dataclass
class VocabShardedSampler:
    """Samples rows whose vocabulary is split contiguously across the ranks of `group`.

    backend="nccl": all-gather of the [B, K+1] candidate blocks through NCCL, then the merge.
    backend="p2p": one kernel per rank pushes its block into every rank's receive buffer over
    NVLink (CUDA IPC mappings made once, at the first call, for up to `max_batch` rows), raises a
    flag per row there, waits for its own flags (bounded) and merges; no collective library on the
    data path. The call epoch is a device counter, so the step (two launches, no host state) can be
    captured in a CUDA graph. A row with status FS_ROW_TIMEOUT (5) means a peer's push did not
    arrive in time and the ranks' exchanges are out of step: close() and build a new sampler
    before the next call. Call close() (every rank) before destroying the process group.
    """

    vocab: int
    top_k: int
    group: Optional[dist.ProcessGroup] = None
    ops: object = None
    bf16: bool = True
    backend: str = "nccl"
    max_batch: int = 64
    wait_polls: int = 0

    def __post_init__(self):
        self.world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        self.cols = shard_range(self.vocab, self.world, self.rank)
        lo, hi = self.cols
        if self.top_k > hi - lo:
            # every shard must be able to hold the k best of its columns
            raise ValueError(f"top_k {self.top_k} exceeds the shard width {hi - lo}")
        if self.ops is None:
            self.ops = _default_ops()
        if self.backend not in ("nccl", "p2p"):
            raise ValueError(f"backend must be 'nccl' or 'p2p', got {self.backend!r}")
        self._gathered = None
        self._p2p = None

    def _setup_p2p(self, device):
        """Allocates this rank's buffers, exchanges IPC handles and maps every peer's. Every rank
        reaches every collective here; a failure on any rank raises RuntimeError on all of them."""
        from . import abi

        W, K1 = self.world, self.top_k + 1

        def agree(ok: bool, what: str):
            oks = [None] * W
            dist.all_gather_object(oks, ok, group=self.group)
            if not all(oks):
                raise RuntimeError(f"p2p exchange set-up failed on rank(s) "
                                   f"{[r for r, o in enumerate(oks) if not o]} while {what}")

        own, opened, handles = [], [], None
        try:
            with torch.cuda.device(device):
                try:
                    recv, recv_ptr = abi.ipc_alloc((2, W, self.max_batch, K1), torch.int64)
                    own.append(recv_ptr)
                    flags, flags_ptr = abi.ipc_alloc((2, W, self.max_batch), torch.int32)
                    own.append(flags_ptr)
                    torch.cuda.synchronize(device)
                    mine = (abi.ipc_handle(recv_ptr), abi.ipc_handle(flags_ptr))
                    ok = True
                except Exception:
                    mine, ok = None, False
                handles = [None] * W
                dist.all_gather_object(handles, mine, group=self.group)
                agree(ok and all(h is not None for h in handles), "exporting buffers")
                recv_ptrs, flag_ptrs = [], []
                try:
                    for r in range(W):
                        if r == self.rank:
                            recv_ptrs.append(recv_ptr)
                            flag_ptrs.append(flags_ptr)
                        else:
                            rp = abi.ipc_open(handles[r][0])
                            opened.append(rp)
                            fp = abi.ipc_open(handles[r][1])
                            opened.append(fp)
                            recv_ptrs.append(rp)
                            flag_ptrs.append(fp)
                    ok = True
                except Exception:
                    ok = False
                agree(ok, "mapping peer buffers")
                peer_recv = torch.tensor(recv_ptrs, dtype=torch.int64, device=device)
                peer_flags = torch.tensor(flag_ptrs, dtype=torch.int64, device=device)
        except Exception:
            for ptr in opened:
                abi.ipc_close(ptr)
            dist.barrier(group=self.group)  # no peer still maps this rank's buffers
            for ptr in own:
                abi.ipc_free(ptr)
            raise
        # every rank has mapped every buffer before any rank pushes into one
        dist.barrier(group=self.group)
        # the call epoch lives on the device: the launch reads and advances it, so a step of
        # shard top-k + exchange-merge can be captured in a CUDA graph and replayed
        epoch_counter = torch.zeros(2, dtype=torch.int32, device=device)
        self._p2p = dict(recv=recv, flags=flags, own=(recv_ptr, flags_ptr), opened=opened,
                         peer_recv=peer_recv, peer_flags=peer_flags, epoch_counter=epoch_counter)

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (p2p backend); collective."""
        if self._p2p is None:
            return
        from . import abi

        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no peer still writes into this rank's buffers
        for ptr in self._p2p["opened"]:
            abi.ipc_close(ptr)
        dist.barrier(group=self.group)  # no peer still maps this rank's buffers
        recv_ptr, flags_ptr = self._p2p["own"]
        self._p2p = None
        abi.ipc_free(recv_ptr)
        abi.ipc_free(flags_ptr)

    def local_candidates(self, shard_logits: torch.Tensor) -> torch.Tensor:
        lo, hi = self.cols
        if shard_logits.shape[1] != hi - lo:
            raise ValueError(f"rank {self.rank} holds columns [{lo}, {hi}) but got {shard_logits.shape[1]}")
        return self.ops.shard_candidates(shard_logits, self.top_k, lo, 0)

    def exchange(self, cand: torch.Tensor) -> torch.Tensor:
        """All-gather [B, K+1] candidate words into [world, B, K+1]."""
        B = cand.shape[0]
        if self._gathered is None or self._gathered.shape[1] != B or self._gathered.device != cand.device:
            self._gathered = torch.empty(self.world, B, self.top_k + 1, dtype=cand.dtype, device=cand.device)
        if self.world == 1:
            self._gathered[0].copy_(cand)
        else:
            # flat [world * B, K + 1] output: the layout every backend accepts; viewed as
            # [world, B, K + 1] (rank-major), which is what the merge reads
            flat = self._gathered.view(self.world * B, self.top_k + 1)
            dist.all_gather_into_tensor(flat, cand.contiguous(), group=self.group)
        return self._gathered

    def sample(self, shard_logits: torch.Tensor, top_p: float, *, seed: int, offset: int,
               uniforms: Optional[torch.Tensor] = None, row_base: int = 0, temperature: float = 1.0):
        """Returns (ids [B], status [B]); identical on every rank. temperature: as in
        ``fused.sample`` (the merged candidates' logits / T in fp32 before the softmax)."""
        if self.backend == "p2p":
            B = shard_logits.shape[0]
            if B > self.max_batch:
                raise ValueError(f"batch {B} exceeds max_batch {self.max_batch} of the p2p buffers")
            if self._p2p is None:
                self._setup_p2p(shard_logits.device)
            st = self._p2p
            cand = self.local_candidates(shard_logits)
            return self.ops.tp_merge(cand, self.bf16, self.top_k, top_p, st["recv"], st["flags"], st["peer_recv"],
                                     st["peer_flags"], self.world, self.rank, 0, uniforms, seed, offset,
                                     row_base, self.wait_polls, temperature=temperature,
                                     epoch_counter=st["epoch_counter"])
        gathered = self.exchange(self.local_candidates(shard_logits))
        ids, status = self.ops.merge_sample(gathered, self.bf16, self.top_k, top_p, None, None, uniforms, seed,
                                            offset, row_base, temperature=temperature)
        return ids, status
