"""World-size-2 data-parallel LM step on CPU ranks (gloo), the CPU stand-in of the NCCL path:
each rank takes half of the batch, DistributedDataParallel all-reduces (averages) the gradients
inside backward, and the clipped AdamW step must leave both ranks with the parameters a single
process gets from the whole batch."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _build():
    from atomic_gdn2 import make_cfg
    from atomic_gdn2.training import GDN2LM
    from oracle_blr import make_oracle_blr, prologue_torch
    cfg = make_cfg(bt=64, bc=32, score_bs=64, bs2=32, mb=8)
    return GDN2LM(cfg, d_model=32, n_heads=2, d_head=16, n_layers=2, seed=5,
                  blr_fn=make_oracle_blr(cfg, 0.25), prologue_fn=prologue_torch).double()


def _batch():
    return torch.randint(0, 256, (4, 128), generator=torch.Generator().manual_seed(9))


def _worker(rank, world, port, out_q):
    import sys, pathlib
    root = pathlib.Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "atomic-ops_b200"), str(root / "tests")]
    from torch.nn.parallel import DistributedDataParallel as DDP
    from atomic_gdn2.training import TrainStep, make_optimizer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = _build()
        ddp = DDP(model)
        step = TrainStep(ddp, make_optimizer(model, 1e-2), lr=1e-2, warmup=0, total=10, clip=0.5)
        ids = _batch().chunk(world)[rank]
        loss, gn, ok = step(ids)
        flat = torch.cat([p.detach().flatten() for p in model.parameters()])
        out_q.put((rank, flat.numpy(), float(gn), bool(ok)))   # by value: the rank may exit first
    finally:
        dist.destroy_process_group()


def test_data_parallel_step_equals_single_process():
    import sys, pathlib
    root = pathlib.Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "tests")]
    from atomic_gdn2.training import TrainStep, make_optimizer
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    model = _build()
    step = TrainStep(model, make_optimizer(model, 1e-2), lr=1e-2, warmup=0, total=10, clip=0.5)
    loss, gn, ok = step(_batch())
    ref = torch.cat([p.detach().flatten() for p in model.parameters()])
    for rank, flat, g, k in res:
        flat = torch.from_numpy(flat)
        assert k and abs(g - float(gn)) < 1e-9 * float(gn)
        assert torch.allclose(flat, ref, rtol=0, atol=1e-12), (rank, float((flat - ref).abs().max()))
