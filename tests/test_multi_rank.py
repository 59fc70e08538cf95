"""CPU, world_size 2 (gloo): the row-sharded path gives the same ids as one
process.  Each rank takes its contiguous shard from the C-ABI sharding rule,
samples it with the global-row seeds (the CPU oracle stands in for the device
kernel here), and the ids are gathered with the same helper the benchmark
uses."""
import os
import socket

import numpy as np
import torch.multiprocessing as mp


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def worker(rank, world, port, batch, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist
    import oracle
    from __graft_entry__ import load_package
    pkg = load_package()
    import llama2_cu_b200.multigpu as mg
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = pkg.workloads.topp(rows=batch, vocab=2048)
    begin, count = mg.local_rows(batch, world, rank)
    seeds = pkg.workloads.row_seeds(count, offset=begin)
    ids, _ = oracle.oracle().sample_batch(w["logits"][begin:begin + count], w["temperature"], w["topp"], seeds,
                                          topp_rows=w["topp_rows"][begin:begin + count])
    full = mg.gather_ids(torch.from_numpy(ids), batch, world, rank)
    if rank == 0:
        np.save(os.path.join(out_dir, "ids.npy"), full.numpy())
    dist.destroy_process_group()


def test_two_rank_sharding_matches_single_process(tmp_path, pkg, orc):
    batch, world = 37, 2
    mp.start_processes(worker, args=(world, free_port(), batch, str(tmp_path)), nprocs=world, start_method="spawn")
    got = np.load(tmp_path / "ids.npy")
    w = pkg.workloads.topp(rows=batch, vocab=2048)
    want, _ = orc.sample_batch(w["logits"], w["temperature"], w["topp"], pkg.workloads.row_seeds(batch),
                               topp_rows=w["topp_rows"])
    assert np.array_equal(got, want)
