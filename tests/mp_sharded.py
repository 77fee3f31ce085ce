"""torchrun worker: vocab-sharded sampling, one process per GPU.

Each rank holds its contiguous slice of the config-5 rows (B=128 here,
V=256000), samples through ShardedSampler with the fused peer exchange (CUDA
IPC buffers, NVLink peer stores) and with the NCCL all-gather path, and rank
0 checks the tokens against the oracle on the full rows and the two paths
against each other.  Run by tests/test_gpu_sharded.py."""
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
        P = b.top_p.copy()
        K[:3] = [0, 1, 300]          # a distributed-nucleus row, a greedy row, a full-row-path row
        T[3] = 0.0
        K[4:12] = 0                  # rows without top-k: top_p 1 (the whole-vocabulary draw) and
        P[4:8] = 1.0                 # high-temperature nuclei wider than the candidates
        T[8:12] = 1.5
        v0, v1 = sharded.shard_bounds(V, world, rank)
        part = torch.from_numpy(np.ascontiguousarray(b.logits[:, v0:v1])).cuda()
        results = {}
        # the fused peer exchange (three calls: both record areas) and the
        # all-gather path must give the same tokens
        for mode in ("peer", "nccl"):
            s = sharded.ShardedSampler(V, exchange=mode)
            for call in range(3 if mode == "peer" else 1):
                tok, prob, st = s.sample(part, v0, T, K, P, uniforms=b.uniforms)
                torch.cuda.synchronize()
            # rows 0 and 4-11 (no top-k) finish without logits crossing ranks;
            # row 2 (top_k 300, above the record width) takes the full-row path
            assert s.last_full_rows <= 1 and s.last_nucleus_rows >= 4, (s.last_full_rows, s.last_nucleus_rows)
            assert s.last_exchange == mode
            s.close()
            tok = tok.cpu().numpy()
            # every rank must hold the same tokens
            t_all = [torch.empty(B, dtype=torch.int64, device="cuda") for _ in range(world)]
            dist.all_gather(t_all, torch.from_numpy(tok).cuda())
            same = all(np.array_equal(t.cpu().numpy(), tok) for t in t_all)
            results[mode] = (tok, prob.cpu().numpy(), st.cpu().numpy())
            if rank == 0:
                from parity import compare
                compare(tok, results[mode][1].astype(np.float64), results[mode][2], b.logits, T, K, P,
                        b.uniforms, label=f"{mode} x{world}")
                assert same, f"ranks disagree ({mode})"
        for a, c in zip(results["peer"], results["nccl"]):
            assert np.array_equal(a, c), "peer exchange and all-gather paths disagree"
        if rank == 0:
            print("sharded ok", world, flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
