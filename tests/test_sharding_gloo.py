"""World-size-2 test of the batch x head sharding on CPU ranks (gloo backend).

Each rank runs the CPU oracle on its shard of heads (as the GPU ranks run the operator in
bench.py); the gathered result must equal the unsharded computation exactly, and an uneven split
(B*H not divisible by the world size) must cover every head once.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from atomic_gdn2.sharding import bh_range, gather_heads, shard_heads


def test_bh_range_partitions():
    for B, H, world in ((4, 6, 2), (4, 6, 8), (1, 3, 2), (2, 5, 4)):
        seen = []
        for r in range(world):
            s, e = bh_range(B, H, r, world)
            seen.extend(range(s, e))
        assert seen == list(range(B * H))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, B, H, L, D, out_q):
    import sys, pathlib
    root = pathlib.Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "atomic-ops_b200")]
    from oracle import gdn2_oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        (q, k, v, w, b, g), h0 = O.bench_inputs(B, H, L, D, 7)
        xs = [shard_heads(t.double(), rank, world) for t in (q, k, v, w, b, g)]
        h0s = shard_heads(h0.double(), rank, world)
        cfg = O.OracleCfg(bt=64, score_bs=64, mb=8, wy_eps=0.0)
        o, hf = O.forward_hm(*xs, D ** -0.5, h0s, cfg)
        o_full = gather_heads(o, B, H, world)
        hf_full = gather_heads(hf, B, H, world)
        if rank == 0:
            o_ref, hf_ref = O.forward_hm(*(t.double() for t in (q, k, v, w, b, g)), D ** -0.5, h0.double(), cfg)
            out_q.put((float((o_full - o_ref).abs().max()), float((hf_full - hf_ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B,H", [(2, 3), (1, 3)])
def test_sharded_equals_unsharded_gloo(B, H):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, B, H, 128, 16, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    do, dh = q.get(timeout=10)
    assert do == 0.0 and dh == 0.0
