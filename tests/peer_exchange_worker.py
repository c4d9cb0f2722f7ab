"""Worker of tests/test_gpu_shared_bounds.py: one rank of a 2-GPU row-sharded
exact index exchanging over peer memory (run under torch.distributed.run)."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
from elips_b200.distributed import ShardedExactIndex  # noqa: E402
from tests import helpers as H  # noqa: E402


def main(out_path):
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        n, d = 80_000, 96
        base = H.gaussian(n, d, seed=81)
        base[40_000:40_100] = base[:100]
        queries = torch.from_numpy(H.gaussian(500, d, seed=82)).cuda()
        ix = ShardedExactIndex("euclidean", d, n, precision="fp32", device=local)
        assert ix.exchange == "peer"
        ix.add_device(torch.from_numpy(base[ix.row_begin:ix.row_end]).cuda())
        res = {}
        # a single-query batch first: the buffers are sized for one query, so
        # both sets' layout has to stay aligned for an odd batch size
        d1, r1 = ix.search_device(queries[:1], 20)
        d1b, r1b = ix.search_device(queries[:1], 20)
        torch.cuda.synchronize()
        if dist.get_rank() == 0:
            res["dist1"], res["rows1"] = d1b.cpu().numpy(), r1b.cpu().numpy()
            assert np.array_equal(d1.cpu().numpy(), res["dist1"])
        for k in (10, 100):
            for _ in range(3):          # several steps: both buffer sets, bounds reset between steps
                dd, rr = ix.search_device(queries, k)
            torch.cuda.synchronize()
            if dist.get_rank() == 0:
                res[f"dist{k}"] = dd.cpu().numpy()
                res[f"rows{k}"] = rr.cpu().numpy()
        if dist.get_rank() == 0:
            np.savez(out_path, **res)
        ix.peer.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
