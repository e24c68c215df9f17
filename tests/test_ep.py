"""Expert-parallel exchange logic on CPU ranks (gloo), no GPU.

The local grouped GEMM is replaced by the fp64 C oracle, which computes each
row independently, so the EP result must be bit-identical to the oracle run
on each rank's rows with the full, unsharded B.  A second test drops a rank
and checks that the survivor fails with an error instead of hanging.
"""

import datetime
import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    """A fresh rendezvous file (no TCP port, so no port races between tests)."""
    fd, path = tempfile.mkstemp(prefix="gmm_rdzv_")
    os.close(fd)
    os.unlink(path)
    return path


def _oracle_local_gemm(a, b, bs, trans_b):
    import oracle
    return torch.from_numpy(oracle.gmm_oracle_c(a, b, bs, trans_b).astype("float32"))


def _rank_inputs(rank, E, dim, dim_out, trans_b, skew):
    g = torch.Generator().manual_seed(100 + rank)
    tokens = 40 + 13 * rank
    if skew:  # some experts empty on some ranks, one expert hot
        w = torch.ones(E)
        w[0] = 6.0
        w[(rank + 1) % E] = 0.0
        ids = torch.multinomial(w, tokens, replacement=True, generator=g)
    else:
        ids = torch.randint(0, E, (tokens,), generator=g)
    bs = torch.bincount(ids, minlength=E).to(torch.int64)
    a = torch.randn(int(bs.sum()), dim, generator=g)
    gb = torch.Generator().manual_seed(7)
    shape = (E, dim_out, dim) if trans_b else (E, dim, dim_out)
    b_full = torch.randn(*shape, generator=gb)
    return a, b_full, bs


def _ep_worker(rank, world, port, E, trans_b, skew, chunks):
    import sys
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", init_method=f"file://{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import oracle
        from gmm_b200.ep import ExpertParallelGmm
        dim, dim_out = 24, 40
        a, b_full, bs = _rank_inputs(rank, E, dim, dim_out, trans_b, skew)
        El = E // world
        ep = ExpertParallelGmm(E, local_gemm=_oracle_local_gemm, chunks=chunks)
        try:
            ExpertParallelGmm(world * E + 1, local_gemm=_oracle_local_gemm)
            raise AssertionError("indivisible expert count accepted")
        except ValueError as exc:
            assert "divisible" in str(exc)
        out = ep(a, b_full[rank * El:(rank + 1) * El].contiguous(), bs, trans_b)
        want = torch.from_numpy(oracle.gmm_oracle_c(a, b_full, bs, trans_b).astype("float32"))
        assert out.shape == want.shape
        assert torch.equal(out, want), f"rank {rank}: EP output differs from the oracle"
        # counts exchange and plan agree across ranks
        all_bs = ep.exchange_counts(bs)
        assert all_bs.shape == (world, E) and torch.equal(all_bs[rank], bs)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,E,trans_b,skew,chunks", [
    (2, 8, False, False, 4), (2, 6, True, True, 4), (4, 8, False, True, 4), (3, 3, True, False, 4),
    (2, 8, False, True, 1), (4, 8, True, True, 7), (4, 4, False, False, 3)])
def test_ep_matches_oracle_on_gloo_ranks(world, E, trans_b, skew, chunks):
    """Chunked pipelines with more or fewer chunks than local experts, skewed loads."""
    mp.spawn(_ep_worker, args=(world, _free_port(), E, trans_b, skew, chunks), nprocs=world,
             join=True)


def _dropout_worker(rank, world, port, outdir):
    import sys
    import time
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", init_method=f"file://{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        # this rank leaves between steps: it never joins the exchange
        os._exit(0)
    from gmm_b200.ep import ExpertParallelGmm
    t0 = time.time()
    status = "returned"
    try:
        ep = ExpertParallelGmm(4, local_gemm=_oracle_local_gemm)
        bs = torch.tensor([2, 1, 0, 3])
        ep(torch.randn(6, 8), torch.randn(2, 8, 8), bs)
    except Exception as exc:  # noqa: BLE001
        status = f"raised {type(exc).__name__}"
    with open(os.path.join(outdir, "rank0.txt"), "w") as f:
        f.write(f"{status} {time.time() - t0:.1f}\n")
    os._exit(0)


def test_dropped_rank_is_detected_not_hung():
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_dropout_worker, args=(2, _free_port(), d), nprocs=2, join=False,
                                 start_method="spawn")
        for p in ctx.processes:
            p.join(60)
        alive = [p for p in ctx.processes if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung after its peer left"
        status = open(os.path.join(d, "rank0.txt")).read()
        assert status.startswith("raised"), status


def test_ep_rejects_bad_inputs():
    from gmm_b200.ep import ExpertParallelGmm
    port = _free_port()
    dist.init_process_group("gloo", init_method=f"file://{port}", rank=0, world_size=1)
    try:
        ep = ExpertParallelGmm(4, local_gemm=_oracle_local_gemm)
        with pytest.raises(ValueError, match="Sum of batch_sizes"):
            ep(torch.zeros(5, 8), torch.zeros(4, 8, 8), torch.tensor([1, 1, 1, 1]))
        with pytest.raises(ValueError, match="1D CPU int64"):
            ep.exchange_counts(torch.tensor([1.0, 2.0, 3.0, 4.0]))
        with pytest.raises(ValueError, match="non-negative"):
            ep.exchange_counts(torch.tensor([1, -1, 0, 0]))
        out = ep(torch.ones(3, 8), torch.ones(4, 8, 2), torch.tensor([0, 3, 0, 0]))
        assert torch.equal(out, torch.full((3, 2), 8.0))
    finally:
        dist.destroy_process_group()


def _shm_worker(rank, world, path, outdir):
    import sys
    import time
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", init_method=f"file://{path}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    from gmm_b200.host_exchange import ShmCountExchange
    ex = ShmCountExchange(5, timeout_s=2.0)
    for step in range(3):  # a few steps through both slots
        got = ex(torch.arange(5, dtype=torch.int64) * (rank + 1) + step)
        want = torch.stack([torch.arange(5) * (r + 1) + step for r in range(world)])
        assert torch.equal(got, want), (rank, step, got)
    dist.barrier()
    if rank == 1:
        time.sleep(4)  # never posts the next step
        status = "skipped"
    else:
        try:
            ex(torch.zeros(5, dtype=torch.int64))
            status = "returned"
        except RuntimeError as exc:
            status = "raised " + str(exc)
    with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
        f.write(status)
    dist.barrier()
    ex.close()
    dist.destroy_process_group()


def test_shared_memory_count_exchange_and_its_timeout():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_shm_worker, args=(2, _free_port(), d), nprocs=2, join=True)
        status = open(os.path.join(d, "rank0.txt")).read()
        assert status.startswith("raised") and "did not post" in status, status


def test_balanced_placement_is_a_permutation_that_balances():
    """balanced_placement: a permutation giving every rank E/W experts, and on
    cfg3's Zipf routing (placed by another batch's loads) a far better
    mean/max row ratio than contiguous blocks."""
    from gmm_b200.configs import CONFIGS, batch_sizes_for, history_loads
    from gmm_b200.ep import balanced_placement
    cfg = CONFIGS[3]
    real = batch_sizes_for(cfg)
    perm = balanced_placement(history_loads(cfg), 8)
    assert sorted(perm) == list(range(cfg.num_experts))
    El = cfg.num_experts // 8
    rows = torch.stack([real[perm[r * El:(r + 1) * El]].sum() for r in range(8)]).double()
    contiguous = real.view(8, El).sum(1).double()
    assert rows.mean() / rows.max() > 0.95 > contiguous.mean() / contiguous.max()
    with pytest.raises(ValueError):
        balanced_placement([1, 2, 3], 2)
