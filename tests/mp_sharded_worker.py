"""Worker for tests/test_gpu_multi.py (launched with torchrun, one rank per GPU):
runs the column-sharded GEMM with both gather strategies and checks every rank's
full C against the CPU oracle on sampled rows.  Exits non-zero on mismatch."""
import ctypes
import datetime
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [REPO, os.path.join(REPO, "ojasx-open-source-cuda-_b200"), os.path.join(REPO, "tests")]

import numpy as np
import torch
import torch.distributed as dist

from gpu_helpers import oracle_gemm, rel_l2
from torchcl import _lib as L
from torchcl.mesh import ShardedGemm, column_range


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    lib = L.lib()
    L.check(lib.ojx_init(local, ctypes.byref(L.DeviceInfo())))
    failures = 0
    for (M, N, K) in [(512, 1024, 512), (16, 2048, 1024), (300, 4096, 256)]:
        g = torch.Generator().manual_seed(M + N + K)
        A = torch.randn(M, K, generator=g).bfloat16()
        W = (torch.randn(K, N, generator=g) * 0.05).bfloat16()
        bias = (torch.randn(N, generator=g) * 0.1).bfloat16()
        c0, c1 = column_range(N, world, rank)
        Ad = A.cuda()
        Wd = W[:, c0:c1].contiguous().cuda()
        bd = bias[c0:c1].contiguous().cuda()
        rows = np.array([0, M // 3, M - 1])
        ref = oracle_gemm(A, W, operand=bias, kind="row", unary=("relu",), rows=rows)[rows]
        for strategy in ("p2p", "nccl"):
            sg = ShardedGemm(M, N, K, "bf16", strategy=strategy)
            sg.run(Ad.data_ptr(), Wd.data_ptr(), bd.data_ptr(), ("relu",))
            torch.cuda.synchronize()
            C = sg.c_view().float().cpu().numpy()
            err = rel_l2(C[rows], ref)
            route = L.ROUTES[lib.ojx_last_route()]
            if err > 4e-3:
                print(f"rank {rank} {strategy} {M}x{N}x{K} route={route}: rel-L2 {err:.3e}", flush=True)
                failures += 1
            dist.barrier()
            sg.close()
    t = torch.tensor([failures], device="cuda")
    dist.all_reduce(t)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print(f"sharded GEMM: {world} ranks, failures={int(t.item())}", flush=True)
    return 1 if int(t.item()) else 0


if __name__ == "__main__":
    sys.exit(main())
