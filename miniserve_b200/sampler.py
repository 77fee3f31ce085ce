"""GPU token sampler with miniserve's sampler interface.

``Sampler.sample`` keeps the signature and results of miniserve's
``Sampler.sample(logits, *, temperature, top_k, top_p, seed) -> int``
(miniserve/sampler.py:23-68): greedy at temperature 0, temperature scaling,
top-k, softmax, top-p and an index-order inverse-CDF draw of
``random.Random(seed).random()``.  ``Sampler.sample_batch`` is the batched
form the engine's ``sample_fn(out, plan)`` seam calls (miniserve/overlap.py:
109-112): one token per row of a [B, V] device tensor, per-row parameters,
caller-supplied uniforms for reproducibility, and an optional allowed-token
bitmask that applies the logits-processor hook's -inf convention
(miniserve/model_runner.py:214).

All work runs in ``libmssample.so`` on the tensor's CUDA device, on the
current torch stream.  There is no CPU path: without the library or a CUDA
device every call raises.
"""
from __future__ import annotations

import random
from typing import Optional, Sequence, Tuple, Union

from . import _lib

Number = Union[int, float]


def uniform_for_seed(seed: Optional[int]) -> float:
    """The uniform miniserve draws for a request (miniserve/sampler.py:32,62)."""
    return random.Random(seed).random()


def _torch():
    import torch
    return torch


def _param(x, B: int, dtype, device):
    torch = _torch()
    if isinstance(x, torch.Tensor):
        t = x.to(device=device, dtype=dtype)
        if t.dim() == 0:
            t = t.expand(B)
        if t.shape != (B,):
            raise ValueError(f"per-row parameter has shape {tuple(t.shape)}, expected ({B},)")
        return t.contiguous()
    if isinstance(x, (int, float)):
        return torch.full((B,), x, dtype=dtype, device=device)
    t = torch.as_tensor(list(x), dtype=dtype)
    if t.shape != (B,):
        raise ValueError(f"per-row parameter has {t.numel()} entries, expected {B}")
    return t.to(device)


def check_mask(mask, B: int, V: int, device) -> Tuple[int, int]:
    """(pointer, row stride in words) of an allowed-token bitmask, after the
    checks the kernels rely on: a CUDA int32/uint32 tensor on the logits'
    device, [B, >= ceil(V/32)] with unit column stride (the kernels read
    32-bit words at row * stride)."""
    torch = _torch()
    if not isinstance(mask, torch.Tensor) or mask.dtype not in (torch.int32, torch.uint32) or not mask.is_cuda:
        raise TypeError("mask must be a CUDA int32/uint32 tensor")
    if mask.device != device:
        raise ValueError(f"mask is on {mask.device}, logits on {device}")
    if mask.dim() != 2 or mask.shape[0] != B or mask.shape[1] * 32 < V or mask.stride(1) != 1:
        raise ValueError("mask must be [B, >= ceil(V/32)] with unit column stride")
    return mask.data_ptr(), mask.stride(0)


def check_out(out, B: int, device):
    """Caller-supplied (tokens int64, probs float32, status int32) buffers: each
    a contiguous [B] tensor on the logits' device (the kernel writes them
    through raw pointers)."""
    torch = _torch()
    try:
        tokens, probs, status = out
    except (TypeError, ValueError):
        raise TypeError("out must be a (tokens, probs, status) tuple") from None
    for name, t, dt in (("tokens", tokens, torch.int64), ("probs", probs, torch.float32),
                        ("status", status, torch.int32)):
        if not isinstance(t, torch.Tensor) or t.dtype != dt:
            raise TypeError(f"out {name} must be a {dt} tensor")
        if t.device != device or t.shape != (B,) or not t.is_contiguous():
            raise ValueError(f"out {name} must be a contiguous [{B}] tensor on {device}")
    return tokens, probs, status


class Sampler:
    """Convert logit scores to token ids on the GPU (miniserve/sampler.py:20-68).

    ``path="fast"`` (default) uses the streaming kernel (one CTA per row, the
    row read from HBM once, a second L2 pass for top-p-only rows);
    ``path="generic"`` forces the multi-pass kernel (no vocabulary limit; the
    cross-check of the fast path).  Both give the same results.
    """

    def __init__(self, path: str = "fast") -> None:
        if path not in ("fast", "generic"):
            raise ValueError("path must be 'fast' or 'generic'")
        self.path = path

    def sample(self, logits, *, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
               seed: Optional[int] = None) -> int:
        """One row; same arguments, result and errors as the reference.

        ``logits`` is a 1-D CUDA tensor (fp32/bf16) or a sequence of floats,
        which is copied to the current CUDA device as fp32 (exact for values
        taken from fp32/bf16 logits, which is what miniserve passes).
        """
        torch = _torch()
        if isinstance(logits, torch.Tensor):
            row = logits.reshape(1, -1)
            if not row.is_cuda:
                row = row.to("cuda")
        else:
            row = torch.tensor([list(logits)], dtype=torch.float32, device="cuda")
        if row.dtype not in (torch.float32, torch.bfloat16):
            row = row.float()
        tok, _, st = self.sample_batch(row, temperature=temperature, top_k=top_k, top_p=top_p,
                                       uniforms=[uniform_for_seed(seed)])
        status = int(st[0])
        if status & _lib.MS_ROW_ALL_MASKED:
            raise ZeroDivisionError("float division by zero")
        if status & _lib.MS_ROW_BAD_TEMPERATURE:
            raise ValueError(f"temperature {temperature!r} is outside the supported domain "
                             "(0 for greedy, or a finite positive value)")
        return int(tok[0])

    def sample_batch(self, logits, temperature: Union[Number, Sequence, "object"] = 1.0,
                     top_k: Union[int, Sequence, "object"] = 0,
                     top_p: Union[Number, Sequence, "object"] = 1.0,
                     uniforms=None, seeds: Optional[Sequence[Optional[int]]] = None,
                     mask=None, out=None) -> Tuple["object", "object", "object"]:
        """Sample one token per row of ``logits`` [B, V] (CUDA, fp32 or bf16).

        Per-row parameters may be scalars, sequences or tensors.  ``uniforms``
        ([B] float64) default to ``Random(seeds[b]).random()``.  ``mask`` is an
        optional [B, ceil(V/32)] int32/uint32 bitmask (bit set = allowed).
        Returns ``(tokens int64, probs float32, status int32)`` device tensors;
        ``status`` carries the MS_ROW_* bits of include/mssample.h.
        """
        torch = _torch()
        if not isinstance(logits, torch.Tensor) or not logits.is_cuda:
            raise TypeError("sample_batch needs a CUDA tensor of logits")
        if logits.dim() != 2:
            raise ValueError("logits must be [B, V]")
        if logits.dtype == torch.float32:
            dtype = _lib.MS_DTYPE_F32
        elif logits.dtype == torch.bfloat16:
            dtype = _lib.MS_DTYPE_BF16
        else:
            raise TypeError(f"logits dtype {logits.dtype} is not float32 or bfloat16")
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        B, V = logits.shape
        dev = logits.device
        T = _param(temperature, B, torch.float64, dev)
        K = _param(top_k, B, torch.int32, dev)
        P = _param(top_p, B, torch.float64, dev)
        if uniforms is None:
            seeds = [None] * B if seeds is None else list(seeds)
            if len(seeds) != B:
                raise ValueError("need one seed per row")
            uniforms = [uniform_for_seed(s) for s in seeds]
        U = _param(uniforms, B, torch.float64, dev)
        mask_ptr, mask_ld = None, 0
        if mask is not None:
            mask_ptr, mask_ld = check_mask(mask, B, V, dev)
        if out is None:
            tokens = torch.empty(B, dtype=torch.int64, device=dev)
            probs = torch.empty(B, dtype=torch.float32, device=dev)
            status = torch.empty(B, dtype=torch.int32, device=dev)
        else:
            tokens, probs, status = check_out(out, B, dev)
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev).cuda_stream
            fn = _lib.lib().ms_sample if self.path == "fast" else _lib.lib().ms_sample_generic
            rc = fn(logits.data_ptr(), dtype, B, V, logits.stride(0), T.data_ptr(),
                                      K.data_ptr(), P.data_ptr(), U.data_ptr(), mask_ptr, mask_ld,
                                      tokens.data_ptr(), probs.data_ptr(), status.data_ptr(), stream)
        _lib.check(rc, "ms_sample")
        return tokens, probs, status
