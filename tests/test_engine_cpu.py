"""Host side of the engine seam: per-request parameters with
CompletionRequest's field names and defaults (miniserve/protocol.py:20-33)."""
from dataclasses import dataclass

from miniserve_b200.engine import request_params


@dataclass
class _Req:
    prompt: str = ""
    max_tokens: int = 16
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    seed: int = None


def test_request_params_from_objects_and_mappings():
    assert request_params(_Req()) == (1.0, 0, 1.0, None)
    assert request_params(_Req(temperature=0.7, top_p=0.9, top_k=50, seed=3)) == (0.7, 50, 0.9, 3)
    assert request_params({"temperature": 0, "top_k": 1}) == (0.0, 1, 1.0, None)
    assert request_params({}) == (1.0, 0, 1.0, None)
