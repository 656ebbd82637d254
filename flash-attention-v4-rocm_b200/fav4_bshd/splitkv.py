"""Long-context split-KV attention across GPUs (one process per GPU).

BASELINE's long-context case (B1 H8 S131072, causal) splits the key/value
sequence over G ranks. Every rank holds the full Q, K, V (they are inputs of
the job) and computes, for every query row, the partial attention of its own
keys with fav4_bshd_forward_partial. Partials are merged by the LSE-weighted
combine kernel (fav4_bshd_combine): rank r owns the output rows
[r*Sq/G, (r+1)*Sq/G) and its combine kernel reads that row slice of every
rank's partial directly from the peer's memory over NVLink (plain loads
through torch symmetric memory). No collective moves the data.

Causal masking makes contiguous KV slices very unequal in work, so the KV
sequence is cut into 2G chunks of whole 128-key tiles and rank g takes chunks
g and 2G-1-g (zigzag); each rank merges its two chunk partials locally first.

The host-side pieces (chunking, row ownership) are pure functions so they can
be tested with CPU (gloo) ranks against the oracle.
"""
from __future__ import annotations

import math

BLOCK_N = 128  # keys per K/V tile of the kernel


def zigzag_chunks(sk: int, world: int, rank: int, block: int = BLOCK_N) -> list[tuple[int, int]]:
    """The KV ranges [begin, end) rank `rank` attends: chunks rank and
    2*world-1-rank of 2*world near-equal chunks of whole `block`-key tiles.
    Empty ranges are dropped (very short sequences)."""
    tiles = (sk + block - 1) // block
    n = 2 * world
    bounds = [min(sk, (tiles * c // n) * block) for c in range(n + 1)]
    out = []
    for c in (rank, n - 1 - rank):
        if bounds[c + 1] > bounds[c]:
            out.append((bounds[c], bounds[c + 1]))
    return out


def owned_rows(sq: int, world: int, rank: int) -> tuple[int, int]:
    """Output rows [r0, r1) owned by `rank` (contiguous, near-equal)."""
    per = (sq + world - 1) // world
    r0 = min(sq, rank * per)
    return r0, min(sq, r0 + per)


def causal_work(ranges: list[tuple[int, int]], sq: int) -> int:
    """(row, key) pairs a rank computes under top-left causal masking: key c
    is seen by the rows r with c <= r < sq."""
    total = 0
    for b, e in ranges:
        lo, hi = b, min(e, sq)
        if hi > lo:  # sum_{c=lo}^{hi-1} (sq - c)
            n = hi - lo
            total += n * sq - (lo + hi - 1) * n // 2
    return total


def contiguous_chunk(sk: int, world: int, rank: int, block: int = BLOCK_N) -> tuple[int, int]:
    """Keys [begin, end) of `rank` when the keys are cut into `world` contiguous
    chunks of whole `block`-key tiles (the last ones may be short or empty).
    Balanced for decode-like steps, where every query row sees every key."""
    tiles = (sk + block - 1) // block
    per = (tiles + world - 1) // world
    begin = min(sk, rank * per * block)
    return begin, min(sk, begin + per * block)


class DecodeSplitKV:
    """Decode-like step (a few query rows, a long key cache) across the G GPUs
    of a process group.

    Rank r attends one contiguous chunk of the keys (`contiguous_chunk`) for
    every query row, split again inside one kernel launch so that its own GPU
    is filled (fav4_bshd_forward_partial_splitkv), and writes the chunk's
    partial O and LSE to torch symmetric memory. After a device barrier every
    rank's combine kernel reads all G partials for all rows directly from the
    peers' memory over NVLink (plain loads) and writes the full output, so each
    rank ends with the whole O [B, Sq, H, 128] and LSE [B, H, Sq]; a second
    barrier keeps the partials alive until every rank has read them. No
    collective moves data. For causal masking (top-left) the chunks are not
    balanced; decode steps attend the whole cache.
    """

    def __init__(self, group, batch: int, heads: int, sq: int, sk: int, device, causal: bool = False,
                 config: int = 0, splits: int = 0):
        import ctypes as C
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        import fav4_bshd
        self.torch = torch
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.b, self.h, self.sq, self.sk = batch, heads, sq, sk
        self.causal, self.config = causal, config
        self.runner = fav4_bshd.Runner()
        self.kv = contiguous_chunk(sk, self.world, self.rank)
        n = self.kv[1] - self.kv[0]
        if splits == 0 and n > 0:
            a = fav4_bshd.Args(16, 32, 48, 64, 80, batch, heads, sq, n, 1.0)
            splits = max(1, self.runner.lib.fav4_bshd_splitkv_splits(C.byref(a), int(causal), config))
        self.splits = max(1, splits)
        self.o_part = symm.empty((batch, sq, heads, 128), dtype=torch.bfloat16, device=device)
        self.lse_part = symm.empty((batch, heads, sq), dtype=torch.float32, device=device)
        self.o_hdl = symm.rendezvous(self.o_part, group)
        self.l_hdl = symm.rendezvous(self.lse_part, group)
        self.out_o = torch.empty((batch, sq, heads, 128), dtype=torch.bfloat16, device=device)
        self.out_l = torch.empty((batch, heads, sq), dtype=torch.float32, device=device)

    def partials(self, q, k, v):
        """This rank's chunk: partial O and LSE of every query row."""
        if self.kv[1] <= self.kv[0]:
            self.o_part.zero_()
            self.lse_part.fill_(-math.inf)
        else:
            self.runner.call_partial_splitkv(q, k, v, self.o_part, self.lse_part, self.causal, self.kv[0],
                                             self.kv[1], self.config, self.splits)

    def exchange_and_combine(self):
        import ctypes as C
        self.o_hdl.barrier(channel=0)
        stream = self.torch.cuda.current_stream().cuda_stream
        o_ptrs = (C.c_void_p * self.world)(*[self.o_hdl.buffer_ptrs[g] for g in range(self.world)])
        l_ptrs = (C.c_void_p * self.world)(*[self.l_hdl.buffer_ptrs[g] for g in range(self.world)])
        status = self.runner.lib.fav4_bshd_combine(o_ptrs, l_ptrs, self.world, self.out_o.data_ptr(),
                                                   self.out_l.data_ptr(), self.b, self.h, self.sq, stream)
        if status:
            raise RuntimeError(f"combine: CUDA status {status}")
        self.o_hdl.barrier(channel=1)
        return self.out_o, self.out_l

    def forward(self, q, k, v):
        self.partials(q, k, v)
        return self.exchange_and_combine()


class SplitKV:
    """Split-KV forward over a process group of GPUs.

    Buffers are allocated once per shape:
    * this rank's merged partial O [B, Sq, H, 128] (BF16) in symmetric memory;
    * its partial LSE re-laid as [G, B, H, Sq/G] in symmetric memory, so the
      row slice owned by rank r is contiguous.
    forward() returns this rank's output rows: O [B, Sq/G, H, 128] and
    LSE [B, H, Sq/G].
    """

    def __init__(self, group, batch: int, heads: int, sq: int, sk: int, device):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        import fav4_bshd
        self.torch = torch
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if sq % self.world:
            raise ValueError(f"sq={sq} must be a multiple of the group size {self.world}")
        self.b, self.h, self.sq, self.sk = batch, heads, sq, sk
        self.runner = fav4_bshd.Runner()
        self.rows = sq // self.world
        self.r0, self.r1 = owned_rows(sq, self.world, self.rank)
        self.ranges = zigzag_chunks(sk, self.world, self.rank)
        self.o_part = symm.empty((batch, sq, heads, 128), dtype=torch.bfloat16, device=device)
        self.lse_xchg = symm.empty((self.world, batch, heads, self.rows), dtype=torch.float32, device=device)
        self.o_hdl = symm.rendezvous(self.o_part, group)
        self.l_hdl = symm.rendezvous(self.lse_xchg, group)
        self.chunk_o = [torch.empty((batch, sq, heads, 128), dtype=torch.bfloat16, device=device)
                        for _ in self.ranges]
        self.chunk_l = [torch.empty((batch, heads, sq), dtype=torch.float32, device=device) for _ in self.ranges]
        self.lse_full = torch.empty((batch, heads, sq), dtype=torch.float32, device=device)
        self.out_o = torch.empty((batch, self.rows, heads, 128), dtype=torch.bfloat16, device=device)
        self.out_l = torch.empty((batch, heads, self.rows), dtype=torch.float32, device=device)

    def partials(self, q, k, v, causal: bool, config: int = 0):
        """Attention of every query row to this rank's keys, merged into the
        symmetric buffers."""
        if not self.ranges:
            self.o_part.zero_()
            self.lse_full.fill_(-math.inf)
        else:
            for (b, e), o, l in zip(self.ranges, self.chunk_o, self.chunk_l):
                self.runner.call_partial(q, k, v, o, l, causal, b, e, config)
            self.runner.combine(self.chunk_o, self.chunk_l, self.o_part, self.lse_full)
        self.lse_xchg.copy_(self.lse_full.view(self.b, self.h, self.world, self.rows).permute(2, 0, 1, 3))

    def exchange_and_combine(self):
        """Device barrier, then this rank's combine kernel reads its rows of
        every peer's partial over NVLink; a second barrier keeps peers from
        overwriting their partials while they are still being read."""
        import ctypes as C
        self.o_hdl.barrier(channel=0)
        stream = self.torch.cuda.current_stream().cuda_stream
        for bi in range(self.b):
            o_ptrs = [self.o_hdl.buffer_ptrs[g] + ((bi * self.sq + self.r0) * self.h * 128) * 2
                      for g in range(self.world)]
            l_ptrs = [self.l_hdl.buffer_ptrs[g] + ((self.rank * self.b + bi) * self.h * self.rows) * 4
                      for g in range(self.world)]
            status = self.runner.lib.fav4_bshd_combine(
                (C.c_void_p * self.world)(*o_ptrs), (C.c_void_p * self.world)(*l_ptrs), self.world,
                self.out_o[bi].data_ptr(), self.out_l[bi].data_ptr(), 1, self.h, self.rows, stream)
            if status:
                raise RuntimeError(f"combine: CUDA status {status}")
        self.o_hdl.barrier(channel=1)
        return self.out_o, self.out_l

    def forward(self, q, k, v, causal: bool, config: int = 0):
        self.partials(q, k, v, causal, config)
        return self.exchange_and_combine()
