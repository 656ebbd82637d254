"""World-size-2 CPU (gloo) test of the multi-GPU split-KV host logic.

Each rank takes its zigzag KV chunks (fav4_bshd.splitkv.zigzag_chunks),
computes the kernel-faithful partials with the oracle emulation, merges its
chunks locally, exchanges the partials (a gloo all_gather stands in for the
NVLink peer reads of the GPU path), combines the rows it owns (owned_rows),
and rank 0 checks the gathered rows against the FP64 reference.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from fav4_bshd import splitkv as S
from oracle import ref_attention as R


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, causal, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b, h, sq, sk = 1, 2, 512, 512
        q, k, v = R.inputs(b, h, sq, sk, "normal", seed=21)
        ranges = S.zigzag_chunks(sk, world, rank)
        parts = [R.emulate(q, k, v, causal, kv_begin=a, kv_end=e) for a, e in ranges]
        o_loc, l_loc = R.combine([p[0] for p in parts], [p[1] for p in parts])
        gathered = [None] * world
        dist.all_gather_object(gathered, (o_loc.astype(np.float32), l_loc.astype(np.float32)))
        r0, r1 = S.owned_rows(sq, world, rank)
        o_rows, l_rows = R.combine([g[0][:, r0:r1] for g in gathered], [g[1][:, :, r0:r1] for g in gathered])
        rows = [None] * world
        dist.all_gather_object(rows, (r0, o_rows, l_rows))
        if rank == 0:
            rows.sort(key=lambda t: t[0])
            o = np.concatenate([x[1] for x in rows], axis=1)
            lse = np.concatenate([x[2] for x in rows], axis=2)
            ref, ref_lse = R.reference(q, k, v, causal)
            result.put(R.errors(o.transpose(0, 2, 1, 3), lse, ref, ref_lse))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("causal", [False, True])
def test_split_kv_two_cpu_ranks_match_reference(causal):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, causal, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    stats = q.get(timeout=10)
    assert stats["max_abs"] < 2e-2


@pytest.mark.parametrize("world", [2, 4, 8])
def test_zigzag_chunks_cover_and_balance(world):
    sk = 131072
    ranges = [S.zigzag_chunks(sk, world, r) for r in range(world)]
    cover = sorted(x for rr in ranges for x in rr)
    assert cover[0][0] == 0 and cover[-1][1] == sk
    assert all(a[1] == b[0] for a, b in zip(cover, cover[1:]))
    assert all(a % 128 == 0 for a, _ in cover)
    work = [S.causal_work(rr, sk) for rr in ranges]
    assert min(work) / max(work) > 0.99
    brute = sum(max(0, sk - c) for b, e in ranges[0] for c in range(b, e))
    assert brute == work[0]
    rows = [S.owned_rows(sk, world, r) for r in range(world)]
    assert rows[0][0] == 0 and rows[-1][1] == sk and all(a[1] == b[0] for a, b in zip(rows, rows[1:]))


def test_zigzag_short_sequences_drop_empty_chunks():
    for world in (2, 4, 8):
        cover = sorted(x for r in range(world) for x in S.zigzag_chunks(100, world, r))
        assert cover and cover[0][0] == 0 and cover[-1][1] == 100
        assert all(e > b for b, e in cover)


def test_oracle_combine_handles_empty_parts():
    o = np.ones((1, 3, 1, 128))
    lse = np.array([[[-np.inf, 0.0, 1.0]]])
    oc, lc = R.combine([o, 2 * o], [lse, lse])
    assert np.all(oc[0, 0] == 0) and np.isneginf(lc[0, 0, 0])
    np.testing.assert_allclose(oc[0, 1:], 1.5)
    np.testing.assert_allclose(lc[0, 0, 1:], [np.log(2.0), 1.0 + np.log(2.0)])


def _decode_rank_main(rank, world, port, result):
    """Decode layout: one contiguous key chunk per rank, all query rows; every
    rank combines every peer's partial for all rows (the all_gather stands in
    for the NVLink peer reads of DecodeSplitKV)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b, h, sq, sk = 1, 2, 16, 1000
        q, k, v = R.inputs(b, h, sq, sk, "normal", seed=23)
        kb, ke = S.contiguous_chunk(sk, world, rank)
        if ke > kb:
            o_p, l_p = R.emulate(q, k, v, False, kv_begin=kb, kv_end=ke)
        else:
            o_p, l_p = np.zeros((b, sq, h, 128)), np.full((b, h, sq), -np.inf)
        gathered = [None] * world
        dist.all_gather_object(gathered, (o_p.astype(np.float32), l_p.astype(np.float32)))
        o, lse = R.combine([g[0] for g in gathered], [g[1] for g in gathered])
        ref, ref_lse = R.reference(q, k, v, False)
        result.put((rank, R.errors(o.transpose(0, 2, 1, 3), lse, ref, ref_lse)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_decode_split_kv_cpu_ranks_match_reference(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decode_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = sorted(q.get(timeout=10) for _ in range(world))
    assert [r for r, _ in got] == list(range(world))
    assert all(stats["max_abs"] < 2e-2 for _, stats in got)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_contiguous_chunks_cover(world):
    for sk in (1, 100, 128, 1000, 131072):
        ch = [S.contiguous_chunk(sk, world, r) for r in range(world)]
        assert ch[0][0] == 0 and ch[-1][1] == sk
        assert all(a[1] == b[0] for a, b in zip(ch, ch[1:]))
        assert all(b % 128 == 0 or b == sk for b, _ in ch)
        sizes = [e - b for b, e in ch]
        assert max(sizes) - min(sizes) <= 128 * ((sk + 127) // 128 // world + 1)
