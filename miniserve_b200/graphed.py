"""Sampling inside the decode step's CUDA graph, from its static logits buffer.

miniserve's ``GraphedDecodeRunner`` replays a captured decode step that writes
one static ``[max_batch, V]`` fp32 buffer, ``_out`` (miniserve/model_runner.py:
264-265, written at :277), and returns ``self._out[:B].detach().clone()``
(:321); the sampler then reads the clone (and the reference's ``Sampler``
converts it to Python floats).  ``GraphedSampler`` samples ``_out[:bucket]``
where it lies, as the last launches of the same captured graph: the logits are
neither copied nor read back, and a step hands the host ``B`` tokens (8 bytes
each) instead of ``B * V * 4`` bytes of logits.

The per-row parameters live in static device buffers that the graph reads on
every replay; ``set_params`` writes them before the replay (rows at and past
``B`` in the bucket -- the runner's padding rows -- become greedy rows, the
cheapest mode, and their tokens are ignored).  ``ms_sample`` allocates
nothing and launches only kernels on the capturing stream, which is what
stream capture needs.
"""
from __future__ import annotations

from typing import Optional, Sequence

from . import _lib
from .sampler import _torch, check_mask, uniform_for_seed


class GraphedSampler:
    """Static-buffer sampler for a captured decode graph.

    ``logits``: the graph's static ``[max_batch, V]`` CUDA buffer (fp32 or
    bf16, unit column stride).  ``with_mask``: keep a static allowed-token
    bitmask ``[max_batch, ceil(V/32)]`` (all allowed until ``set_mask``).

    Inside ``torch.cuda.graph(g)``, after the code that writes the logits,
    call ``enqueue(bucket)``; before each ``g.replay()`` call
    ``set_params(B, ...)``; after it ``result(B)`` gives the device tensors
    ``(tokens i64, probs f32, status i32)`` and ``tokens(B)`` the host list.
    ``enqueue`` also works outside a capture (an eager step on the same
    buffers).
    """

    def __init__(self, logits, with_mask: bool = False, path: str = "fast") -> None:
        torch = _torch()
        if not isinstance(logits, torch.Tensor) or not logits.is_cuda or logits.dim() != 2:
            raise TypeError("logits must be the graph's static [max_batch, V] CUDA tensor")
        if logits.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError(f"logits dtype {logits.dtype} is not float32 or bfloat16")
        if logits.stride(1) != 1:
            raise ValueError("logits must have unit column stride (the buffer is read in place)")
        if path not in ("fast", "generic"):
            raise ValueError("path must be 'fast' or 'generic'")
        self.logits = logits
        self.path = path
        self.max_batch, self.V = logits.shape
        dev = logits.device
        self.device = dev
        n = self.max_batch
        self.temperature = torch.zeros(n, dtype=torch.float64, device=dev)
        self.top_k = torch.zeros(n, dtype=torch.int32, device=dev)
        self.top_p = torch.ones(n, dtype=torch.float64, device=dev)
        self.uniforms = torch.zeros(n, dtype=torch.float64, device=dev)
        self.out_tokens = torch.zeros(n, dtype=torch.int64, device=dev)
        self.out_probs = torch.zeros(n, dtype=torch.float32, device=dev)
        self.out_status = torch.zeros(n, dtype=torch.int32, device=dev)
        self.mask = None
        if with_mask:
            self.mask = torch.full((n, (self.V + 31) // 32), -1, dtype=torch.int32, device=dev)
            check_mask(self.mask, n, self.V, dev)
        # the library's one-time per-device setup (a kernel attribute) runs
        # here, outside any capture
        self.enqueue(1)
        torch.cuda.synchronize(dev)

    def set_params(self, B: int, temperature=1.0, top_k=0, top_p=1.0, uniforms=None,
                   seeds: Optional[Sequence[Optional[int]]] = None) -> None:
        """Write rows [0, B) of the static parameters (scalars or length-B
        sequences, ``uniforms`` defaulting to ``Random(seed).random()``) and
        make rows [B, max_batch) greedy.  Host values are copied on the
        current stream, so a replay queued after this call sees them."""
        torch = _torch()
        if not 0 <= B <= self.max_batch:
            raise ValueError(f"B={B} outside [0, {self.max_batch}]")

        def col(x, dtype):
            if isinstance(x, (int, float)):
                v = [x] * B
            elif isinstance(x, torch.Tensor):
                v = x.detach().to("cpu", dtype).reshape(-1).tolist()
            else:
                v = list(x)
            if len(v) != B:
                raise ValueError(f"per-row parameter has {len(v)} entries, expected {B}")
            return v

        if uniforms is None:
            s = [None] * B if seeds is None else list(seeds)
            if len(s) != B:
                raise ValueError("need one seed per row")
            uniforms = [uniform_for_seed(x) for x in s]
        pad = self.max_batch - B
        T = col(temperature, torch.float64) + [0.0] * pad
        K = col(top_k, torch.int32) + [0] * pad
        P = col(top_p, torch.float64) + [1.0] * pad
        U = col(uniforms, torch.float64) + [0.5] * pad
        # pageable host sources: each copy has taken its data when it returns
        self.temperature.copy_(torch.tensor(T, dtype=torch.float64))
        self.top_k.copy_(torch.tensor(K, dtype=torch.int32))
        self.top_p.copy_(torch.tensor(P, dtype=torch.float64))
        self.uniforms.copy_(torch.tensor(U, dtype=torch.float64))

    def set_mask(self, mask) -> None:
        """Copy an allowed-token bitmask ``[b, ceil(V/32)]`` (b <= max_batch)
        into the static mask's first b rows; the rest allow every token."""
        if self.mask is None:
            raise RuntimeError("constructed without with_mask")
        b = mask.shape[0]
        check_mask(mask, b, self.V, self.device)
        self.mask[:b].copy_(mask[:, : self.mask.shape[1]])
        self.mask[b:].fill_(-1)

    def enqueue(self, bucket: int) -> None:
        """Launch the sampling of rows [0, bucket) of the static buffers on the
        current stream (inside a graph capture: as nodes of the graph)."""
        torch = _torch()
        if not 1 <= bucket <= self.max_batch:
            raise ValueError(f"bucket={bucket} outside [1, {self.max_batch}]")
        dtype = _lib.MS_DTYPE_F32 if self.logits.dtype == torch.float32 else _lib.MS_DTYPE_BF16
        mask_ptr, mask_ld = (self.mask.data_ptr(), self.mask.stride(0)) if self.mask is not None else (None, 0)
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            fn = _lib.lib().ms_sample if self.path == "fast" else _lib.lib().ms_sample_generic
            rc = fn(self.logits.data_ptr(), dtype, bucket, self.V, self.logits.stride(0),
                    self.temperature.data_ptr(), self.top_k.data_ptr(), self.top_p.data_ptr(),
                    self.uniforms.data_ptr(), mask_ptr, mask_ld, self.out_tokens.data_ptr(),
                    self.out_probs.data_ptr(), self.out_status.data_ptr(), stream)
        _lib.check(rc, "ms_sample")

    def result(self, B: int):
        """(tokens i64, probs f32, status i32) device views of rows [0, B)."""
        return self.out_tokens[:B], self.out_probs[:B], self.out_status[:B]

    def tokens(self, B: int):
        """The first B tokens on the host (waits for the current stream)."""
        return self.out_tokens[:B].tolist()
