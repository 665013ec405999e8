"""torchrun helper for test_sharded_gpu.py: ShardedIndex over NCCL matches the
CPU oracle on the global corpus and equals a single-GPU Index (rank 0 checks)."""

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
        from helpers import assert_topk_exact
        from oracle import exact_topk

        whole = cvs.Index(x.to(dev), metric="cosine")
        x32 = whole.embeddings.float().cpu().numpy()  # the stored (normalised) global corpus
        q32 = whole._prep_queries(q.to(dev))[:, :d].float().cpu().numpy()
        for kk, (vv, ii) in ((k, (v, i)), (1024, (v2, i2))):
            ov, oi = exact_topk(q32, x32, kk + 1)
            assert_topk_exact(vv.cpu().numpy(), ii.cpu().numpy(), q32, x32, ov, oi, kk)
            ref_v, ref_i = whole.search(q.to(dev), kk)
            assert torch.equal(ii, ref_i), "ids differ from the single-GPU index"
            assert torch.allclose(vv, ref_v, atol=1e-6, rtol=0)
        print("SHARDED OK", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
