"""torchrun helper for test_sharded_gpu.py: ShardedIndex over NCCL equals a
single-GPU Index on the same global corpus (rank 0 checks)."""

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    import cuda_vector_search as cvs

    g = torch.Generator().manual_seed(7)
    n, d, b, k = 40000, 384, 300, 16
    x = torch.randn(n, d, generator=g).half()
    q = torch.randn(b, d, generator=g).half()
    bounds = [round(r * n / world) for r in range(world + 1)]
    idx = cvs.ShardedIndex(x[bounds[rank]:bounds[rank + 1]].to(dev), metric="cosine", device=dev)
    assert idx.row_offset == bounds[rank] and idx.n_total == n
    v, i = idx.search(q.to(dev), k)
    v2, i2 = idx.search(q.to(dev), 1024)
    if rank == 0:
        ref_v, ref_i = cvs.Index(x.to(dev), metric="cosine").search(q.to(dev), k)
        assert torch.equal(i, ref_i), "ids differ"
        assert torch.allclose(v, ref_v, atol=1e-6, rtol=0)
        ref_v2, ref_i2 = cvs.Index(x.to(dev), metric="cosine").search(q.to(dev), 1024)
        assert torch.equal(i2, ref_i2) and torch.allclose(v2, ref_v2, atol=1e-6, rtol=0)
        print("SHARDED OK", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
