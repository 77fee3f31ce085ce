"""Adapters for miniserve's logits-processor hook.

miniserve installs ``fn(logits: Tensor[V], generated: List[int]) -> Tensor[V]``
with ``ModelRunner.set_logits_processor`` (miniserve/model_runner.py:166-168)
and, in ``generate_greedy``, takes ``int(fn(logits, generated).argmax())``
(model_runner.py:214-216); the hook's convention is that a disallowed token's
logit is -inf.  The sampler here takes the allowed set as a bitmask.  These
helpers connect the two without changing either side: the hook still runs
(per row, as miniserve calls it), its output becomes the bitmask on the GPU
(``ms_mask_from_logits``), and the argmax or the sampling runs in the library.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

from . import _lib
from .sampler import Sampler, _torch, check_out


def allowed_mask(processed, out=None):
    """[B, ceil(V/32)] int32 bitmask (bit t & 31 of word t >> 5 set = token t
    allowed) from a hook's output: ``processed`` [B, V] or [V], a CUDA fp32 or
    bf16 tensor; a token is allowed unless its logit is -inf (a NaN counts as
    allowed and the sampler flags the row MS_ROW_NONFINITE)."""
    torch = _torch()
    if not isinstance(processed, torch.Tensor) or not processed.is_cuda:
        raise TypeError("allowed_mask needs a CUDA tensor")
    x = processed.reshape(1, -1) if processed.dim() == 1 else processed
    if x.dim() != 2:
        raise ValueError("hook output must be [V] or [B, V]")
    if x.dtype == torch.float32:
        dtype = _lib.MS_DTYPE_F32
    elif x.dtype == torch.bfloat16:
        dtype = _lib.MS_DTYPE_BF16
    else:
        x, dtype = x.float(), _lib.MS_DTYPE_F32
    if x.stride(1) != 1:
        x = x.contiguous()
    B, V = x.shape
    W = (V + 31) // 32
    if out is None:
        out = torch.empty((B, W), dtype=torch.int32, device=x.device)
    elif out.dtype not in (torch.int32, torch.uint32) or out.shape[0] != B or out.shape[1] < W or out.stride(1) != 1 \
            or out.device != x.device:
        raise ValueError(f"out must be a [{B}, >= {W}] int32 tensor with unit column stride on {x.device}")
    with torch.cuda.device(x.device):
        rc = _lib.lib().ms_mask_from_logits(x.data_ptr(), dtype, B, V, x.stride(0), out.data_ptr(), out.stride(0),
                                            torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(rc, "ms_mask_from_logits")
    return out


def argmax_tokens(logits, out=None):
    """First maximal index of each row of ``logits`` [B, V] (or [V]) on the
    GPU: the temperature-0 path of the sampler, which is torch.argmax's
    first-index rule.  (A NaN is where the two part: torch.argmax returns the
    NaN's index, the sampler reads NaN as -inf and sets MS_ROW_NONFINITE.)"""
    torch = _torch()
    x = logits.reshape(1, -1) if logits.dim() == 1 else logits
    B = x.shape[0]
    if out is not None:
        out = check_out(out, B, x.device)
    tok, _, _ = Sampler().sample_batch(x, temperature=0.0, uniforms=torch.zeros(B, dtype=torch.float64,
                                                                                device=x.device), out=out)
    return tok


class HookAdapter:
    """An installed hook ``fn(logits[V], generated) -> logits[V]`` used with
    the GPU sampler.

    ``greedy(logits, generated)`` is the drop-in for ``generate_greedy``'s
    ``int(fn(logits, generated).argmax())``; ``mask(logits, generated)``
    gives the bitmask of a batch (the hook called per row, as miniserve
    calls it); ``sample_batch(logits, generated, ...)`` samples the raw
    logits under that mask, which is what sampling the hook's output gives.
    """

    def __init__(self, fn: Optional[Callable] = None, sampler: Optional[Sampler] = None) -> None:
        self.fn = fn or (lambda logits, generated: logits)  # ModelRunner.set_logits_processor(None)
        self.sampler = sampler or Sampler()

    def processed(self, logits, generated: Sequence[List[int]]):
        """The hook applied to each row of ``logits`` [B, V]: [B, V]."""
        torch = _torch()
        if logits.dim() == 1:
            return self.fn(logits, list(generated)).reshape(1, -1)
        if len(generated) != logits.shape[0]:
            raise ValueError("need one generated-token list per row")
        return torch.stack([self.fn(logits[b], list(generated[b])) for b in range(logits.shape[0])])

    def mask(self, logits, generated: Sequence[List[int]]):
        return allowed_mask(self.processed(logits, generated))

    def greedy(self, logits, generated: List[int]) -> int:
        """``int(fn(logits, generated).argmax())`` for one [V] row."""
        return int(argmax_tokens(self.fn(logits, list(generated)))[0])

    def sample_batch(self, logits, generated: Sequence[List[int]], **params):
        """``Sampler.sample_batch`` on the raw ``logits`` [B, V] with the
        hook's allowed set as the mask."""
        return self.sampler.sample_batch(logits, mask=self.mask(logits, generated), **params)
