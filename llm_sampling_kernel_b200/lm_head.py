"""Sampling straight from the LM head: ``logits = hidden @ weight.T`` is produced in vocabulary
chunks and each chunk is consumed by the shard top-k kernel while it is still in L2, so the
``[B, V]`` logits never go to HBM and back.

Per call, for each chunk ``[c0, c1)`` of the vocabulary:

1. a bf16 GEMM (cuBLAS, through ``torch.matmul``) writes ``hidden @ weight[c0:c1].T`` into one of
   two L2-sized staging buffers (about 32 MB each);
2. ``shard_candidates`` reads that chunk (an L2 hit: the GEMM has just written it) and writes the
   chunk's top-K as packed (order key, global id) words plus the chunk's row status into part
   ``c`` of a ``[parts, B, K + 1]`` block.

Then ``merge_sample`` merges the ``parts * K`` candidates of every row and samples with the usual
tail -- the same machinery as vocabulary-sharded tensor parallelism, with the chunks of one GPU as
the shards. The ids equal the plain sampler's over the concatenated chunk logits (the merge of
exact per-shard top-Ks is the exact top-K), which the tests check.

HBM traffic per call: the weight (V * H * 2 bytes) and the hidden states, plus B * parts * (K + 1)
* 8 bytes of candidates; the unfused pipeline adds a B * V * 2 byte logits write and read, and a
[B, V] logits buffer.

Measured on B200 (B=1024, H=4096, V=151936, k=50): the GEMM alone takes about 870 µs; the GEMM
writing [B, V] logits to HBM followed by one sampler call about 930-960 µs; this pipeline about
1240 µs. Ten per-chunk top-k calls at B=1024 cost more than the 311 MB round trip they avoid, so
the pipeline's gain is memory (no [B, V] logits buffer), not time; saving time needs the selection
inside the GEMM's epilogue.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops as _ops

L2_CHUNK_BYTES = 32 << 20  # one staging buffer: a quarter of the B200's 126 MB L2


class LMHeadSampler:
    """Samples token ids from ``hidden [B, H] @ weight[V, H].T`` (bf16) without materialising the
    ``[B, V]`` logits in HBM.

    top_k is the bound K of every call (at most 8192 // parts candidates survive into the merge,
    where parts = ceil(V / chunk)); chunk defaults to the largest multiple of 256 columns whose
    ``[max_batch, chunk]`` bf16 block fits L2_CHUNK_BYTES.
    """

    def __init__(self, weight: torch.Tensor, top_k: int, *, max_batch: int = 1024, chunk: Optional[int] = None,
                 ops=None):
        if weight.dim() != 2 or weight.dtype != torch.bfloat16 or not weight.is_cuda:
            raise ValueError("weight must be a bf16 cuda [V, H] tensor")
        self.weight = weight.contiguous()
        self.vocab, self.hidden = self.weight.shape
        self.top_k = int(top_k)
        self.max_batch = int(max_batch)
        if chunk is None:
            chunk = max(256, (L2_CHUNK_BYTES // (2 * self.max_batch)) // 256 * 256)
        self.chunk = int(min(chunk, self.vocab))
        self.bounds = [(c0, min(c0 + self.chunk, self.vocab)) for c0 in range(0, self.vocab, self.chunk)]
        if len(self.bounds) > 1 and self.bounds[-1][1] - self.bounds[-1][0] < top_k:
            # a tail narrower than top_k joins the chunk before it
            self.bounds[-2:] = [(self.bounds[-2][0], self.vocab)]
        if self.top_k < 1 or any(hi - lo < self.top_k for lo, hi in self.bounds):
            raise ValueError(f"top_k {self.top_k} must be >= 1 and fit every chunk of {self.chunk} columns")
        if len(self.bounds) * self.top_k > 8192:
            raise ValueError(f"{len(self.bounds)} chunks x top_k {self.top_k} exceed the merge's 8192 candidates")
        self.ops = ops if ops is not None else _ops()
        dev = self.weight.device
        # two staging buffers: chunk c + 1's GEMM (caller's stream) runs while chunk c's top-k
        # (a side stream) reads the other buffer; events order each buffer's reuse
        width = max(hi - lo for lo, hi in self.bounds)
        self._stage = [torch.empty(self.max_batch * width, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self._side = torch.cuda.Stream(device=dev)
        self._ready = [torch.cuda.Event() for _ in range(2)]
        self._free = [torch.cuda.Event() for _ in range(2)]

    @property
    def parts(self) -> int:
        return len(self.bounds)

    def chunk_logits(self, hidden: torch.Tensor, c: int) -> torch.Tensor:
        """The logits of chunk c, ``hidden @ weight[c0:c1].T`` ([B, c1 - c0] bf16, in a staging
        buffer that the next call of chunk c + 2 overwrites)."""
        lo, hi = self.bounds[c]
        B = hidden.shape[0]
        out = self._stage[c % 2][: B * (hi - lo)].view(B, hi - lo)
        torch.matmul(hidden, self.weight[lo:hi].t(), out=out)
        return out

    def candidates(self, hidden: torch.Tensor) -> torch.Tensor:
        """The ``[parts, B, K + 1]`` candidate block: every chunk's top-K packed words and status."""
        if hidden.dim() != 2 or hidden.shape[1] != self.hidden or hidden.dtype != torch.bfloat16:
            raise ValueError(f"hidden must be a bf16 [B, {self.hidden}] tensor")
        B = hidden.shape[0]
        if B > self.max_batch:
            raise ValueError(f"batch {B} exceeds max_batch {self.max_batch}")
        cand = torch.empty(self.parts, B, self.top_k + 1, dtype=torch.int64, device=hidden.device)
        main = torch.cuda.current_stream(hidden.device)
        self._side.wait_stream(main)  # hidden, cand and the staging buffers are ready
        for c, (lo, _) in enumerate(self.bounds):
            i = c % 2
            if c >= 2:
                main.wait_event(self._free[i])  # chunk c - 2's top-k has read this buffer
            logits = self.chunk_logits(hidden, c)
            self._ready[i].record(main)
            self._side.wait_event(self._ready[i])
            with torch.cuda.stream(self._side):
                self.ops.shard_candidates(logits, self.top_k, lo, 0, out=cand[c])
            self._free[i].record(self._side)
        main.wait_stream(self._side)  # the merge reads every part
        cand.record_stream(self._side)
        return cand

    def sample(self, hidden: torch.Tensor, top_p: float, *, seed: int = 0, offset: int = -1,
               uniforms: Optional[torch.Tensor] = None, temperature: float = 1.0):
        """(ids [B] int64, status [B] int32) for ``hidden [B, H]``; offset < 0 draws from torch's
        default CUDA generator (graph-safe), as ``fused.sample_fused`` does."""
        cand = self.candidates(hidden)
        return self.ops.merge_sample(cand, True, self.top_k, float(top_p), None, None, uniforms, int(seed),
                                     int(offset), 0, float(temperature))
