"""The engine's sampling seam: ``sample_fn(out, plan) -> tokens``.

miniserve's ``OverlapEngine`` (and ``LLMEngine`` on top of it) calls
``sample_fn(out, plan)`` on its sampling thread with the forward's output for
the plan's batch rows and returns one token per row, in row order
(miniserve/overlap.py:109-112, ``StepPlan.row_rids`` at overlap.py:35-41).
``make_sample_fn`` builds that callable on top of ``Sampler.sample_batch``:
each row's parameters come from its request (``temperature``, ``top_k``,
``top_p``, ``seed`` as in ``CompletionRequest``, miniserve/protocol.py:20-33),
and the sampling runs on a side CUDA stream, so it overlaps the next forward
pass on the engine's stream.
"""
from __future__ import annotations

from typing import Any, Callable, Dict, List, Mapping, Optional, Tuple, Union

from .sampler import Sampler, _torch, uniform_for_seed

Params = Tuple[float, int, float, Optional[int]]  # (temperature, top_k, top_p, seed)


def request_params(req: Any) -> Params:
    """(temperature, top_k, top_p, seed) of a request object or mapping with
    ``CompletionRequest``'s field names and defaults."""
    get = (lambda k, d: req.get(k, d)) if isinstance(req, Mapping) else (lambda k, d: getattr(req, k, d))
    return (float(get("temperature", 1.0)), int(get("top_k", 0)), float(get("top_p", 1.0)), get("seed", None))


class SampleFn:
    """``sample_fn(out, plan) -> list[int]`` for ``OverlapEngine``.

    ``params``: rid -> request (or a (temperature, top_k, top_p, seed) tuple),
    as a mapping or a callable.  ``out``: the forward's logits for the plan's
    rows, a [B, V] (or [V] for one row) fp32/bf16 tensor, or a sequence of
    per-row float sequences.  ``mask_fn(out, plan)`` may return an allowed-token
    bitmask [B, ceil(V/32)] (e.g. ``JsonMaskBuilder.build``).  With
    ``side_stream`` the kernel runs on a stream of its own that first waits for
    the work already queued on the caller's stream (the forward that produced
    ``out``); the call returns once the tokens are on the host.
    """

    def __init__(self, params: Union[Mapping[str, Any], Callable[[str], Any]], sampler: Optional[Sampler] = None,
                 side_stream: bool = True, mask_fn: Optional[Callable[[Any, Any], Any]] = None) -> None:
        self._params = params
        self._sampler = sampler if sampler is not None else Sampler()
        self._mask_fn = mask_fn
        self._use_side = side_stream
        self._streams: Dict[int, Any] = {}
        self.last = None  # (tokens, probs, status) device tensors of the last call

    def _lookup(self, rid: str) -> Params:
        p = self._params(rid) if callable(self._params) else self._params[rid]
        if isinstance(p, tuple) and len(p) == 4:
            return (float(p[0]), int(p[1]), float(p[2]), p[3])
        return request_params(p)

    def _logits(self, out):
        torch = _torch()
        if isinstance(out, torch.Tensor):
            x = out if out.dim() == 2 else out.reshape(1, -1)
            if not x.is_cuda:
                x = x.to("cuda")
        else:
            x = torch.tensor([list(r) for r in out], dtype=torch.float32, device="cuda")
        if x.dtype not in (torch.float32, torch.bfloat16):
            x = x.float()
        return x

    def __call__(self, out, plan) -> List[int]:
        torch = _torch()
        x = self._logits(out)
        rids = list(plan.row_rids)
        if len(rids) != x.shape[0]:
            raise ValueError(f"plan has {len(rids)} rows, the logits {x.shape[0]}")
        rows = [self._lookup(rid) for rid in rids]
        T = [r[0] for r in rows]
        K = [r[1] for r in rows]
        P = [r[2] for r in rows]
        U = [uniform_for_seed(r[3]) for r in rows]
        mask = self._mask_fn(out, plan) if self._mask_fn is not None else None
        caller = torch.cuda.current_stream(x.device)
        if self._use_side:
            side = self._streams.get(x.device.index)
            if side is None:
                side = self._streams[x.device.index] = torch.cuda.Stream(device=x.device)
            side.wait_stream(caller)  # the forward that wrote the logits
            with torch.cuda.stream(side):
                res = self._sampler.sample_batch(x, T, K, P, uniforms=U, mask=mask)
                # the inputs were made on the caller's stream: keep them alive
                # until the side stream is done with them
                x.record_stream(side)
                if mask is not None:
                    mask.record_stream(side)
                tok = res[0].to("cpu", non_blocking=False)
        else:
            res = self._sampler.sample_batch(x, T, K, P, uniforms=U, mask=mask)
            tok = res[0].cpu()
        self.last = res
        return [int(t) for t in tok.tolist()]


def make_sample_fn(params, sampler: Optional[Sampler] = None, side_stream: bool = True,
                   mask_fn=None) -> SampleFn:
    """``sample_fn`` for ``OverlapEngine(scheduler, forward_fn, sample_fn)`` /
    ``LLMEngine(..., sample_fn)``; see :class:`SampleFn`."""
    return SampleFn(params, sampler=sampler, side_stream=side_stream, mask_fn=mask_fn)
