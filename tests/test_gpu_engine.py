"""The engine seam ``sample_fn(out, plan)`` (miniserve/overlap.py:109-112):
per-request parameters by rid, side-stream sampling, the tokens of
``Sampler.sample_batch`` in plan row order.  Needs a B200."""
from dataclasses import dataclass, field
from typing import Dict, List

import numpy as np
import pytest

from parity import compare

pytestmark = pytest.mark.gpu


@dataclass
class _Plan:  # the fields of miniserve's StepPlan that sample_fn reads
    rows: List[List[int]]
    row_rids: List[str]
    ev: Dict = field(default_factory=dict)


@dataclass
class _Req:  # CompletionRequest's sampling fields
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    seed: int = None


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    if not t.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return t


@pytest.mark.parametrize("side", [True, False])
def test_sample_fn_matches_sample_batch_and_oracle(torch, side):
    from miniserve_b200 import workloads
    from miniserve_b200.engine import make_sample_fn
    from miniserve_b200.sampler import uniform_for_seed
    b = workloads.config3(3, B=24)
    rids = [f"r{i}" for i in range(24)]
    reqs = {rid: _Req(float(b.temperature[i]), float(b.top_p[i]), int(b.top_k[i]), 1000 + i)
            for i, rid in enumerate(rids)}
    order = np.random.default_rng(1).permutation(24)  # plan rows in another order
    plan = _Plan(rows=[[0]] * 24, row_rids=[rids[i] for i in order])
    x = torch.from_numpy(b.logits[order]).cuda()
    fn = make_sample_fn(reqs, side_stream=side)
    toks = fn(x, plan)
    U = np.array([uniform_for_seed(1000 + int(i)) for i in order])
    tok = np.array(toks)
    prob = fn.last[1].cpu().numpy().astype(np.float64)
    st = fn.last[2].cpu().numpy()
    compare(tok, prob, st, b.logits[order], b.temperature[order], b.top_k[order], b.top_p[order], U,
            label="sample_fn")


def test_sample_fn_list_logits_and_tuples(torch):
    from miniserve_b200 import Sampler
    from miniserve_b200.engine import make_sample_fn
    rng = np.random.default_rng(4)
    logits = rng.normal(0, 2, (3, 500)).astype(np.float32)
    params = {"a": (0.0, 0, 1.0, None), "b": (0.8, 20, 0.9, 7), "c": (1.2, 0, 0.7, 8)}
    fn = make_sample_fn(lambda rid: params[rid])
    toks = fn(logits.tolist(), _Plan(rows=[[0]] * 3, row_rids=["a", "b", "c"]))
    s = Sampler()
    want = [s.sample(logits[i].tolist(), temperature=p[0], top_k=p[1], top_p=p[2], seed=p[3])
            for i, p in enumerate(params.values())]
    assert toks == want
