"""Multi-process host logic of the batch-sharded bench on CPU (gloo, world size 2):
weights synchronised from rank 0, distinct per-rank input shards, an all-gather of the logits
equal to a single-process forward of the concatenated batch, and max-over-ranks timing.
The forward is the bench's CPU reference arm (the reference's own modules with the SRNL
recurrence on the oracle port), so no GPU is needed."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        import bench

        ref, model = bench.reference_cpu_model("visionhope_tiny", depths=(1, 1, 1, 1), num_classes=10)
        if rank:
            torch.manual_seed(100 + rank)  # a different local init on purpose
            for p in model.parameters():
                p.data.normal_(0, 0.02)
        bench.sync_model(model, world)
        x = bench.rank_inputs(1, rank, torch.device("cpu"))
        with bench.oracle_srnl(ref), torch.inference_mode():
            logits = model(x)
        gathered = [torch.empty_like(logits) for _ in range(world)]
        dist.all_gather(gathered, logits)
        ms = bench.max_over_ranks(10.0 + rank, torch.device("cpu"), world)
        if rank == 0:
            torch.save({"gathered": torch.cat(gathered), "ms": ms,
                        "state": {k: v.clone() for k, v in model.state_dict().items()},
                        "inputs": torch.cat([bench.rank_inputs(1, r, torch.device("cpu")) for r in range(world)])},
                       os.path.join(out_dir, "rank0.pt"))
    finally:
        dist.destroy_process_group()


def test_two_rank_batch_sharding(tmp_path):
    from oracle import refmodel

    if not refmodel.available():
        pytest.skip("reference package not staged (oracle/build_ref.py stage_python)")
    world, port = 2, _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    res = torch.load(tmp_path / "rank0.pt")
    assert res["ms"] == 11.0
    import bench

    ref, model = bench.reference_cpu_model("visionhope_tiny", depths=(1, 1, 1, 1), num_classes=10)
    model.load_state_dict(res["state"])
    assert not torch.equal(res["inputs"][0], res["inputs"][1])
    with bench.oracle_srnl(ref), torch.inference_mode():
        ref = model(res["inputs"].contiguous(memory_format=torch.channels_last))
    torch.testing.assert_close(res["gathered"], ref, rtol=1e-4, atol=1e-5)
