"""JSON-grammar allowed-token masks on the GPU.

``allowed[b][t] = is_valid_prefix(prefix_b + vocab[t])`` for miniserve's
``JSONLogitsProcessor.is_valid_prefix`` (miniserve/sampler.py:139-148), the
``allowed_token_ids(partial, vocab)`` the reference names at sampler.py:120.
Each row keeps a parse state on the device (``init`` from the prefixes,
``advance`` by the token just sampled); ``build`` evaluates every token of the
vocabulary against it and returns the [B, ceil(V/32)] bitmask that
``Sampler.sample_batch(..., mask=...)`` applies.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

from . import _lib
from .sampler import _torch

ROW_RAISES = 1      # some token makes the reference raise (its bit is 0)
ROW_TOKEN_DEEP = 2  # some token opens/closes more than 64 containers beyond the row's (its bit is 0)


def _pack_texts(texts: Sequence[str], device):
    torch = _torch()
    blobs = [t.encode("utf-8") for t in texts]
    off = [0]
    for b in blobs:
        off.append(off[-1] + len(b))
    data = b"".join(blobs) or b"\0"
    by = torch.frombuffer(bytearray(data), dtype=torch.uint8).to(device)
    return by, torch.tensor(off, dtype=torch.int64, device=device)


def _plain(b: bytes) -> bool:
    """A short token with no '"', '\\' or control byte: it leaves a JSON string
    body a string body (the mask kernel settles it without the automaton)."""
    return 0 < len(b) <= 16 and all(c >= 0x20 and c not in (0x22, 0x5C) for c in b)


def length_order(vocab: Sequence[str]) -> List[int]:
    """Token ids sorted by (plain first, UTF-8 length, bytes): a warp of the
    mask kernel then holds tokens of one length that share their first bytes,
    so its lanes take the same automaton steps and finish together, and rows
    inside a string settle whole warps of plain tokens at once."""
    enc = [t.encode("utf-8") for t in vocab]
    return sorted(range(len(enc)), key=lambda t: (not _plain(enc[t]), len(enc[t]), enc[t]))


class JsonMaskBuilder:
    """Masks over a fixed vocabulary (a list of token strings).

    ``order``: "length" (default) evaluates the tokens in ``length_order``
    (``ms_build_json_mask_ordered``); None keeps token order
    (``ms_build_json_mask_packed``).  The masks are the same either way."""

    def __init__(self, vocab: Sequence[str], device="cuda", order: Optional[str] = "length") -> None:
        torch = _torch()
        if order not in (None, "length"):
            raise ValueError(f"order must be 'length' or None, not {order!r}")
        self.device = torch.device(device)
        self.V = len(vocab)
        self.vocab_bytes, self.vocab_off = _pack_texts(vocab, self.device)
        self.words = int(_lib.lib().ms_json_state_words())
        # fixed-width copy of the vocabulary (16 bytes a token) for the mask
        self.packed = torch.empty((self.V, 4), dtype=torch.int32, device=self.device)
        self.lens = torch.empty(self.V, dtype=torch.uint8, device=self.device)
        self.order = None
        if order == "length" and self.V > 0:
            self.order = torch.tensor(length_order(vocab), dtype=torch.int32, device=self.device)
            rc = _lib.lib().ms_json_pack_vocab_ordered(self.vocab_bytes.data_ptr(), self.vocab_off.data_ptr(),
                                                       self.V, self.order.data_ptr(), self.packed.data_ptr(),
                                                       self.lens.data_ptr(), self._stream())
            _lib.check(rc, "ms_json_pack_vocab_ordered")
        else:
            rc = _lib.lib().ms_json_pack_vocab(self.vocab_bytes.data_ptr(), self.vocab_off.data_ptr(), self.V,
                                               self.packed.data_ptr(), self.lens.data_ptr(), self._stream())
            _lib.check(rc, "ms_json_pack_vocab")

    def _stream(self):
        return _torch().cuda.current_stream(self.device).cuda_stream

    def init(self, prefixes: Sequence[str]):
        """Parse states [B, words] (int32) after each row's prefix."""
        torch = _torch()
        B = len(prefixes)
        by, off = _pack_texts(prefixes, self.device)
        states = torch.empty((B, self.words), dtype=torch.int32, device=self.device)
        rc = _lib.lib().ms_json_init(by.data_ptr(), off.data_ptr(), B, states.data_ptr(), self._stream())
        _lib.check(rc, "ms_json_init")
        return states

    def advance(self, states, tokens) -> None:
        """Append token tokens[b] (int64 ids, < 0: none) to row b, in place."""
        torch = _torch()
        t = torch.as_tensor(tokens, dtype=torch.int64, device=self.device)
        rc = _lib.lib().ms_json_advance(states.data_ptr(), states.shape[0], self.vocab_bytes.data_ptr(),
                                        self.vocab_off.data_ptr(), self.V, t.data_ptr(), self._stream())
        _lib.check(rc, "ms_json_advance")

    def build(self, states, out=None, packed: bool = True, status=None) -> Tuple["object", "object"]:
        """(mask [B, ceil(V/32)] int32, row_status [B] int32).  packed=False
        reads every token from the variable-length vocabulary instead of the
        fixed-width copy (same result).  ``out`` / ``status``: buffers to
        write into."""
        torch = _torch()
        B = states.shape[0]
        W = (self.V + 31) // 32
        mask = torch.empty((B, W), dtype=torch.int32, device=self.device) if out is None else out
        if status is None:
            status = torch.empty(B, dtype=torch.int32, device=self.device)
        if packed and self.order is not None:
            rc = _lib.lib().ms_build_json_mask_ordered(states.data_ptr(), B, self.vocab_bytes.data_ptr(),
                                                       self.vocab_off.data_ptr(), self.packed.data_ptr(),
                                                       self.lens.data_ptr(), self.order.data_ptr(), self.V,
                                                       mask.data_ptr(),
                                                       mask.stride(0), status.data_ptr(), self._stream())
            _lib.check(rc, "ms_build_json_mask_ordered")
        elif packed:
            rc = _lib.lib().ms_build_json_mask_packed(states.data_ptr(), B, self.vocab_bytes.data_ptr(),
                                                      self.vocab_off.data_ptr(), self.packed.data_ptr(),
                                                      self.lens.data_ptr(), self.V, mask.data_ptr(), mask.stride(0),
                                                      status.data_ptr(), self._stream())
            _lib.check(rc, "ms_build_json_mask_packed")
        else:
            rc = _lib.lib().ms_build_json_mask(states.data_ptr(), B, self.vocab_bytes.data_ptr(),
                                               self.vocab_off.data_ptr(), self.V, mask.data_ptr(), mask.stride(0),
                                               status.data_ptr(), self._stream())
            _lib.check(rc, "ms_build_json_mask")
        return mask, status
