"""Two GPUs (skipped with fewer): each rank samples its contiguous row shard
on its own GPU with the global-row seeds, and the library's NCCL all-gather
(sampler_nccl_*) assembles the ids on every rank; they must equal one GPU
sampling the whole batch."""
import ctypes
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


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
    from __graft_entry__ import load_package
    pkg = load_package()
    L = pkg.lib()
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    w = pkg.workloads.topp(rows=batch)
    begin, count = pkg.shard_rows(batch, world, rank)
    x = torch.from_numpy(w["logits"][begin:begin + count]).cuda()
    tr = torch.from_numpy(w["topp_rows"][begin:begin + count]).cuda()
    st = torch.empty(count, dtype=torch.int64, device="cuda")
    pkg.seed_states(st, 42, begin)
    ids = pkg.sample_batched(x, w["temperature"], w["topp"], st, topp_rows=tr)
    # NCCL id from rank 0, shared over the CPU group
    uid = torch.zeros(128, dtype=torch.uint8)
    if rank == 0:
        assert L.sampler_nccl_get_unique_id(ctypes.c_void_p(uid.data_ptr())) == 0
    dist.broadcast(uid, 0)
    comm = ctypes.c_void_p()
    assert L.sampler_nccl_comm_init(ctypes.byref(comm), world, ctypes.c_void_p(uid.data_ptr()), rank) == 0
    full = torch.empty(batch, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    assert L.sampler_nccl_allgather_ids(comm, ctypes.c_void_p(ids.data_ptr()), count, ctypes.c_void_p(full.data_ptr()),
                                        ctypes.c_void_p(stream.cuda_stream)) == 0
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"ids{rank}.npy"), full.cpu().numpy())
    L.sampler_nccl_comm_destroy(comm)
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_sampling_with_nccl_gather(tmp_path, pkg):
    batch, world = 512, 2
    mp.start_processes(worker, args=(world, free_port(), batch, str(tmp_path)), nprocs=world, start_method="spawn")
    w = pkg.workloads.topp(rows=batch)
    x = torch.from_numpy(w["logits"]).cuda()
    st = torch.empty(batch, dtype=torch.int64, device="cuda")
    pkg.seed_states(st, 42, 0)
    want = pkg.sample_batched(x, w["temperature"], w["topp"], st, topp_rows=torch.from_numpy(w["topp_rows"]).cuda())
    torch.cuda.synchronize()
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"ids{r}.npy"), want.cpu().numpy())
