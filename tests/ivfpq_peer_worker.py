"""Worker of tests/test_gpu_shared_bounds.py: one rank of a 2-GPU list-sharded
IVF-PQ index whose scans share their bounds and whose k best go to the root
over peer memory (run under torch.distributed.run)."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
from elips_b200.distributed import PeerExchange, ShardedIvfPqIndex, balanced_lists  # noqa: E402
from tests import helpers as H  # noqa: E402


def main(out_path):
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        rank, world = dist.get_rank(), dist.get_world_size()
        m = H.ivfpq_tie_model()
        owner = balanced_lists(np.bincount(m["asg"], minlength=len(m["cent"])), world)
        ix = ShardedIvfPqIndex("euclidean", 64, m["cent"], m["cb"], 8, rank=rank, world=world, device=local,
                               owner=owner)
        assert isinstance(ix.peer, PeerExchange)
        ix.add_device(torch.from_numpy(m["base"]).cuda(), torch.from_numpy(m["asg"].view(np.int32)).cuda(), 0,
                      torch.from_numpy(m["codes"]).cuda())
        queries = torch.from_numpy(m["queries"]).cuda()
        res = {}
        for k in (10, 20):
            for nq in (200, 120, 200):   # both buffer sets; a smaller batch between larger ones
                dd, rr = ix.search_device(queries[:nq], k)
            torch.cuda.synchronize()
            if rank == 0:
                res[f"dist{k}"] = dd.cpu().numpy()
                res[f"rows{k}"] = rr.cpu().numpy()
        if rank == 0:
            np.savez(out_path, **res)
        ix.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
