"""Data-parallel host logic on two CPU ranks (gloo): sharding, the bucketed
scan-gradient all-reduce, and failure detection when a rank disappears.

The model math is the CPU oracle of the reference Mamba (no GPU needed); the
reduced gradients of two half-batch ranks must equal the full-batch gradients
of one process.  The failure test makes rank 1 leave before the collective;
rank 0 must get an error from the short process-group timeout, not hang.
"""

import datetime
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from redpanda_b200.distributed import (OverlappedGradAllReducer, ScanGradAllReducer,
                                       SCAN_PARAM_SUFFIXES, shard_rows)

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model_grads(rows_ids, sd, kw):
    from oracle import model_oracle as MO
    cfg = MO.OracleConfig(vocab_size=64, bidirectional=False, **kw)
    p = {k: v.clone().requires_grad_(v.is_floating_point()) for k, v in sd.items()}
    y = MO.model_forward(p, cfg, rows_ids)
    y.pow(2).mean(dim=(1, 2)).mean().backward()
    return p


def _dp_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    c = torch.load(os.path.join(GOLDEN, "model_verify_trk.pt"))
    ids = torch.randint(0, 64, (4, 17))
    a, b = shard_rows(ids.shape[0], rank, world)
    p = _model_grads(ids[a:b], c["state_dict"], c["kw"])
    named = [(k, v) for k, v in p.items() if k.endswith(SCAN_PARAM_SUFFIXES)]
    red = ScanGradAllReducer(params=named)
    red.synchronize()
    torch.save({k: v.grad for k, v in named}, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_shard_rows_covers_batch():
    for n in (1, 7, 8, 1024, 8191):
        for w in (1, 2, 3, 8):
            spans = [shard_rows(n, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(w - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def test_two_rank_allreduce_equals_full_batch():
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_dp_worker, args=(2, port, d), nprocs=2, join=True,
                           start_method="spawn")
        r0 = torch.load(os.path.join(d, "rank0.pt"))
        r1 = torch.load(os.path.join(d, "rank1.pt"))
    torch.manual_seed(0)
    c = torch.load(os.path.join(GOLDEN, "model_verify_trk.pt"))
    ids = torch.randint(0, 64, (4, 17))
    full = _model_grads(ids, c["state_dict"], c["kw"])
    assert set(r0) == set(r1) and len(r0) == 2 * 6   # 2 layers x 6 scan parameters
    for k in r0:
        assert torch.equal(r0[k], r1[k]), k          # every rank holds the same result
        assert torch.allclose(r0[k], full[k].grad, rtol=1e-5, atol=1e-8), k


def _overlap_worker(rank, world, port, out_dir):
    """Two micro-batches per rank; the bucketed all-reduce of every parameter
    gradient is armed for the second backward only (gradient accumulation)."""
    from oracle import model_oracle as MO
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    c = torch.load(os.path.join(GOLDEN, "model_verify_trk.pt"))
    ids = torch.randint(0, 64, (4, 17))
    a, b = shard_rows(ids.shape[0], rank, world)
    cfg = MO.OracleConfig(vocab_size=64, bidirectional=False, **c["kw"])
    p = {k: v.clone().requires_grad_(v.is_floating_point()) for k, v in c["state_dict"].items()}
    red = OverlappedGradAllReducer(params=[v for v in p.values() if v.requires_grad],
                                   bucket_bytes=16 << 10)
    assert len(red.buckets) > 2
    rows = list(range(a, b))
    for i, r in enumerate(rows):
        if i == len(rows) - 1:
            red.arm()
        y = MO.model_forward(p, cfg, ids[r:r + 1])
        (y.pow(2).mean(dim=(1, 2)).sum() / len(rows)).backward()
    red.finish()
    torch.save({k: v.grad for k, v in p.items() if v.requires_grad},
               os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_overlapped_bucketed_allreduce_with_accumulation_equals_full_batch():
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_overlap_worker, args=(2, port, d), nprocs=2, join=True,
                           start_method="spawn")
        r0 = torch.load(os.path.join(d, "rank0.pt"))
        r1 = torch.load(os.path.join(d, "rank1.pt"))
    torch.manual_seed(0)
    c = torch.load(os.path.join(GOLDEN, "model_verify_trk.pt"))
    ids = torch.randint(0, 64, (4, 17))
    full = _model_grads(ids, c["state_dict"], c["kw"])
    assert set(r0) == set(r1) and len(r0) > 12
    for k in r0:
        assert torch.equal(r0[k], r1[k]), k
        assert torch.allclose(r0[k], full[k].grad, rtol=1e-5, atol=1e-8), k


def _fault_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)                                  # leaves between steps, before the collective
    x = torch.ones(8)
    msg = "no error"
    try:
        dist.all_reduce(x)
    except Exception as e:                           # timeout or peer-closed error
        msg = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(msg)
    os._exit(0)


def test_lost_rank_is_detected_not_hung():
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_fault_worker, args=(2, port, d), nprocs=2, join=False,
                                 start_method="spawn")
        ok = ctx.join(timeout=90)
        if not ok:
            ctx.join(timeout=30)
        for p in ctx.processes:
            if p.is_alive():
                p.kill()
                pytest.fail("a rank hung after its peer left")
        with open(os.path.join(d, "rank0.txt")) as f:
            assert f.read().startswith("error")
