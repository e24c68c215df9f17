"""Expert parallelism over NCCL on 2+ GPUs: the EP forward must be
bit-identical to the single-GPU operator applied to each rank's rows with
the full (unsharded) B -- every output row is computed by the same kernel
from the same operands, only its neighbours in the tile differ."""

import datetime
import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    """A fresh rendezvous file (no TCP port, so no port races between tests)."""
    fd, path = tempfile.mkstemp(prefix="gmm_rdzv_")
    os.close(fd)
    os.unlink(path)
    return path


def _worker(rank, world, port, E, dtype, trans_b, transport, tile):
    import sys
    sys.path.insert(0, ROOT)
    if tile != "auto":  # the single-GPU op and the EP layer must run the same kernel family
        from gmm_b200 import capi
        capi.set_tile_kind(tile)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"file://{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from gmm_b200 import hopper_gmm_fwd
        from gmm_b200.ep import ExpertParallelGmm
        dim, dim_out = 512, 768
        g = torch.Generator().manual_seed(1000 + rank)
        w = torch.rand(E, generator=g) + 0.1
        w[(3 * rank) % E] = 0.0  # an expert this rank never routes to
        ids = torch.multinomial(w, 700 + 150 * rank, replacement=True, generator=g)
        bs = torch.bincount(ids, minlength=E).to(torch.int64)
        a = torch.randn(int(bs.sum()), dim, generator=g).to(dtype).to(dev)
        gb = torch.Generator().manual_seed(5)
        shape = (E, dim_out, dim) if trans_b else (E, dim, dim_out)
        b_full = (torch.randn(*shape, generator=gb) / dim ** 0.5).to(dtype).to(dev)
        El = E // world
        ep = ExpertParallelGmm(E, transport=transport)
        b_local = b_full[rank * El:(rank + 1) * El].contiguous()
        want = hopper_gmm_fwd(a, b_full, bs, trans_b=trans_b)
        ep.overlap_min_rows = 0  # overlap the own-rows GEMM with the gather whatever the sizes
        for step in range(3):  # later steps reuse every buffer; the last runs without overlap
            if step == 2:
                ep.overlap = False
            out = ep(a, b_local, bs, trans_b)
            torch.cuda.synchronize()
            assert torch.equal(out, want), f"rank {rank} step {step}: EP differs from the single-GPU op"
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["direct", "nccl"])
@pytest.mark.parametrize("E,dtype,trans_b,tile", [(8, torch.bfloat16, False, "256"),
                                                  (16, torch.float16, True, "128"),
                                                  (8, torch.float32, False, "auto")])
def test_ep_matches_single_gpu(E, dtype, trans_b, tile, transport):
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = min(n, 8)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_worker, args=(world, _free_port(), E, dtype, trans_b, transport, tile), nprocs=world,
             join=True)
