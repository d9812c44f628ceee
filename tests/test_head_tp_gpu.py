"""Head-tensor-parallel decode on 2 GPUs: the fused gather (combine kernel storing into every
rank's output over peer memory) against the single-GPU decode of all heads and against the
NCCL all-gather baseline -- bit for bit.  Two shapes: 24 sessions over an 8-page prefix, and
128 sessions over a 256-page prefix, where the shared-prefix pass cuts the prefix into chunks
longer than its minimum (the chunk must not depend on how many KV heads a rank holds).
Skipped with fewer than 2 GPUs."""
import datetime
import os
import random

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, result):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from loopfuse_b200 import attention as att
        from loopfuse_b200.runtime.head_tp import HeadParallelDecode
        ok_fused = ok_nccl = True
        for N, P, W, NPRE in ((24, 1100, 48, 8), (128, 5400, 296, 256)):
            g = torch.Generator(device="cpu").manual_seed(7 + N)
            Hq, Hkv, D = 32, 8, 128
            k = torch.randn(P, Hkv, 16, D, generator=g).bfloat16().to(dev)
            v = torch.randn(P, Hkv, 16, D, generator=g).bfloat16().to(dev)
            q = torch.randn(N, Hq, D, generator=g).bfloat16().to(dev)
            perm = torch.randperm(P, generator=g)
            prefix, rest = perm[:NPRE], perm[NPRE:]                  # N x (W - NPRE) own pages
            table = torch.stack([torch.cat([prefix, rest[i * (W - NPRE):(i + 1) * (W - NPRE)]])
                                 for i in range(N)]).to(torch.int32).to(dev)
            lens = torch.randint(NPRE * 16 + 1, W * 16, (N,), generator=g).to(torch.int32).to(dev)
            full = att.paged_decode(q, k, v, table, lens, num_prefix_pages=NPRE, pages_per_split=8)
            hk, hq = Hkv // world, Hq // world
            k_loc = k[:, rank * hk:(rank + 1) * hk].contiguous()
            v_loc = v[:, rank * hk:(rank + 1) * hk].contiguous()
            q_loc = q[:, rank * hq:(rank + 1) * hq].contiguous()
            tp = HeadParallelDecode(N, Hq, D, dev)
            for _ in range(3):                                      # both output buffers
                fused = tp.decode(q_loc, k_loc, v_loc, table, lens, num_prefix_pages=NPRE,
                                  pages_per_split=8)
                ok_fused = ok_fused and bool(torch.equal(fused, full))
            base = tp.decode_nccl(q_loc, k_loc, v_loc, table, lens, num_prefix_pages=NPRE,
                                  pages_per_split=8)
            ok_nccl = ok_nccl and bool(torch.equal(base, full))
            torch.cuda.synchronize()
            tp.close()
        result[rank] = (ok_fused, ok_nccl)
    finally:
        dist.destroy_process_group()


def test_head_parallel_decode_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = 29700 + random.randint(0, 200)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    assert dict(result) == {0: (True, True), 1: (True, True)}
