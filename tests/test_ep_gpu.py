"""Expert-parallel MoE on 2+ GPUs (NCCL), compared with the single-GPU layer
on the concatenated tokens. Each output row depends only on its own token and
its experts, and the tcgen05 GEMM's per-row arithmetic does not depend on
which rows share a tile, so the results must agree bit for bit. Skipped when
fewer than 2 GPUs are visible."""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

T, H, E, F, K = 512, 512, 16, 256, 2


def _make(dev):
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    wr = (torch.randn((E, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w13 = (torch.randn((E, 2 * F, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, F), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    return wr, w13, w2


def _tokens(rank, dev):
    g = torch.Generator(device=dev)
    g.manual_seed(100 + rank)
    return torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)


def _worker(rank, world, outdir, overlap=True):
    import torch.distributed as dist
    from kvm_b200.ep import ExpertParallelMoE
    from kvm_b200 import ops
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    # file rendezvous in the test's own directory: no port to race for
    dist.init_process_group("nccl", init_method=f"file://{outdir}/rendezvous", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        wr, w13, w2 = _make(dev)
        layer = ExpertParallelMoE(wr, w13, w2, top_k=K, max_tokens=T, rank=rank, world=world,
                                  overlap=overlap)
        for _ in range(3):   # later calls reuse every buffer (epochs 2, 3)
            out = layer(_tokens(rank, dev))
        ops.device_status()
        torch.save(out.cpu(), os.path.join(outdir, f"out{rank}.pt"))
        layer.close()
    finally:
        dist.destroy_process_group()



@pytest.mark.parametrize("overlap", [True, False])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_matches_single_gpu(world, overlap):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, d, overlap), nprocs=world,
                           start_method="spawn")
        outs = [torch.load(os.path.join(d, f"out{r}.pt")) for r in range(world)]
    from kvm_b200.moe import MoELayer
    dev = torch.device("cuda:0")
    wr, w13, w2 = _make(dev)
    x = torch.cat([_tokens(r, torch.device("cuda", r)).to(dev) for r in range(world)])
    ref = MoELayer(wr, w13, w2, K, T * world)(x).cpu()
    got = torch.cat(outs)
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("overlap", [True, False])
def test_expert_parallel_single_rank_matches_layer(cuda, overlap):
    """world = 1 runs every exchange kernel (flags, counts, dispatch, combine;
    overlapped: prepare, local scatter, the fused dispatch + gate/up and down
    + push GEMMs) on one GPU; no kernel waits on a concurrently running one."""
    from kvm_b200.ep import ExpertParallelMoE
    from kvm_b200.moe import MoELayer
    from kvm_b200 import ops
    wr, w13, w2 = _make(cuda)
    x = _tokens(0, cuda)
    ref = MoELayer(wr, w13, w2, K, T)(x).clone()
    layer = ExpertParallelMoE(wr, w13, w2, top_k=K, max_tokens=T, rank=0, world=1,
                              overlap=overlap)
    for _ in range(3):
        out = layer(x)
    ops.device_status()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    layer.close()
