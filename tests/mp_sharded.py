"""torchrun worker: vocab-sharded sampling over NCCL, one process per GPU.

Each rank holds its contiguous slice of the config-5 rows (B=128 here,
V=256000), samples through ShardedSampler, and rank 0 checks the tokens
against the oracle on the full rows.  Run by tests/test_gpu_sharded.py."""
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    try:
        from miniserve_b200 import sharded, workloads
        b = workloads.config5(5, B=128)
        B, V = b.logits.shape
        K = b.top_k.copy()
        T = b.temperature.copy()
        K[:3] = [0, 1, 300]          # a fallback row, a greedy row, a fallback row
        T[3] = 0.0
        v0, v1 = sharded.shard_bounds(V, world, rank)
        part = torch.from_numpy(np.ascontiguousarray(b.logits[:, v0:v1])).cuda()
        s = sharded.ShardedSampler(V)
        tok, prob, st = s.sample(part, v0, T, K, b.top_p, uniforms=b.uniforms)
        torch.cuda.synchronize()
        tok = tok.cpu().numpy()
        # every rank must hold the same tokens
        t_all = [torch.empty(B, dtype=torch.int64, device="cuda") for _ in range(world)]
        dist.all_gather(t_all, torch.from_numpy(tok).cuda())
        same = all(np.array_equal(t.cpu().numpy(), tok) for t in t_all)
        if rank == 0:
            from parity import compare
            compare(tok, prob.cpu().numpy().astype(np.float64), st.cpu().numpy(), b.logits, T, K, b.top_p,
                    b.uniforms, label=f"nccl x{world}")
            assert same, "ranks disagree"
            print("sharded ok", world, flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
