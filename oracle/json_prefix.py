"""CPU oracle for the JSON-grammar allowed-token mask -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` use this module,
and only as the checker; the mask the product uses is built on the GPU by
``ms_build_json_mask`` (libmssample.so).

The reference's prefix test is ``JSONLogitsProcessor.is_valid_prefix``
(miniserve/sampler.py:139-148): a string is a valid prefix when it is empty,
starts with ``{``, parses with ``json.loads``, or fails with a
``JSONDecodeError`` whose message contains "Expecting" or "Unterminated".
The token mask of a row is ``allowed[t] = is_valid_prefix(prefix + vocab[t])``
(the ``allowed_token_ids(partial, vocab)`` the reference names at
sampler.py:120).  The arithmetic lives in a dependency that is not part of the
reference tree: the CPython standard library ``json`` decoder with its C
scanner (``_json``), pinned by the interpreter, Python 3.12.3.  Which error
``json.loads`` raises first decides the answer:

  "Expecting value", "Expecting ',' delimiter", "Expecting ':' delimiter",
  "Expecting property name enclosed in double quotes",
  "Unterminated string starting at"                         -> True
  "Invalid \\escape", "Invalid \\uXXXX escape",
  "Invalid control character at", "Extra data"              -> False
  no error                                                   -> True

and two non-JSONDecodeError exceptions propagate out of the reference (the
answer here is RAISE): an integer literal of more than 4300 digits (int()
conversion limit) and nesting of 9997 or more containers (RecursionError when
called from a shallow Python stack; the exact depth depends on the caller).

This module restates the C scanner's control flow (scan_once, the array and
object parsers, scanstring, match_number) index by index, with an explicit
container stack instead of recursion.  It is pinned against the live
reference by ``tests/golden/make_json_golden.py`` (committed vectors) and by
``tests/test_json_oracle.py`` (fuzzing, where the reference tree is present).
"""
from __future__ import annotations

from typing import List, Union

RAISE = "raise"
WS = " \t\n\r"
HEX = "0123456789abcdefABCDEF"
MAX_DEPTH = 9996          # containers; the 9997th nested one raises RecursionError
INT_MAX_DIGITS = 4300     # sys.get_int_max_str_digits() default

Answer = Union[bool, str]


class _Decided(Exception):
    def __init__(self, ok: bool) -> None:
        self.ok = ok


class _Raises(Exception):
    pass


def _skip_ws(s: str, idx: int) -> int:
    n = len(s)
    while idx < n and s[idx] in WS:
        idx += 1
    return idx


def _scanstring(s: str, end: int) -> int:
    """Index after the closing quote of the string whose body starts at `end`."""
    n = len(s)
    while True:
        nxt = end
        c = ""
        while nxt < n:
            c = s[nxt]
            if c == '"' or c == "\\":
                break
            if ord(c) <= 0x1F:
                raise _Decided(False)          # Invalid control character at
            nxt += 1
        if nxt >= n:
            raise _Decided(True)               # Unterminated string starting at
        nxt += 1
        if c == '"':
            return nxt
        if nxt == n:
            raise _Decided(True)               # Unterminated string starting at
        c = s[nxt]
        if c != "u":
            if c not in '"\\/bfnrt':
                raise _Decided(False)          # Invalid \escape
            end = nxt + 1
            continue
        nxt += 1
        end = nxt + 4
        if end >= n:                           # the four digits and one more character
            raise _Decided(False)              # Invalid \uXXXX escape
        h = s[nxt:end]
        if any(ch not in HEX for ch in h):
            raise _Decided(False)
        cp = int(h, 16)
        if 0xD800 <= cp <= 0xDBFF and end + 6 < n and s[end] == "\\" and s[end + 1] == "u":
            h2 = s[end + 2:end + 6]
            if any(ch not in HEX for ch in h2):
                raise _Decided(False)
            if 0xDC00 <= int(h2, 16) <= 0xDFFF:
                end += 6


def _number(s: str, idx: int):
    """End index of the number at `idx`, or None (no number: StopIteration)."""
    n = len(s)
    last = n - 1
    start = idx
    if s[idx] == "-":
        idx += 1
        if idx > last:
            return None
    c = s[idx]
    if "1" <= c <= "9":
        idx += 1
        while idx <= last and "0" <= s[idx] <= "9":
            idx += 1
    elif c == "0":
        idx += 1
    else:
        return None
    int_end = idx
    is_float = False
    if idx < last and s[idx] == "." and "0" <= s[idx + 1] <= "9":
        is_float = True
        idx += 2
        while idx <= last and "0" <= s[idx] <= "9":
            idx += 1
    if idx < last and s[idx] in "eE":
        e_start = idx
        idx += 1
        if idx < last and s[idx] in "-+":
            idx += 1
        while idx <= last and "0" <= s[idx] <= "9":
            idx += 1
        if "0" <= s[idx - 1] <= "9":
            is_float = True
        else:
            idx = e_start
    if not is_float:
        digits = int_end - start - (1 if s[start] == "-" else 0)
        if digits > INT_MAX_DIGITS:
            raise _Raises()                    # ValueError from int()
    return idx


def _scan(s: str) -> int:
    """Index after the top-level value (the decoder's raw_decode)."""
    n = len(s)
    stack: List[str] = []
    idx = _skip_ws(s, 0)
    mode = "value"
    while True:
        if mode == "value":
            if idx >= n:
                raise _Decided(True)           # Expecting value
            c = s[idx]
            if c == '"':
                idx = _scanstring(s, idx + 1)
                mode = "after"
            elif c == "{" or c == "[":
                if len(stack) >= MAX_DEPTH:
                    raise _Raises()            # RecursionError
                stack.append(c)
                idx = _skip_ws(s, idx + 1)
                close = "}" if c == "{" else "]"
                if idx < n and s[idx] == close:   # empty container
                    stack.pop()
                    idx += 1
                    mode = "after"
                else:
                    mode = "key" if c == "{" else "value"
            elif c == "n" and s[idx:idx + 4] == "null":
                idx, mode = idx + 4, "after"
            elif c == "t" and s[idx:idx + 4] == "true":
                idx, mode = idx + 4, "after"
            elif c == "f" and s[idx:idx + 5] == "false":
                idx, mode = idx + 5, "after"
            elif c == "N" and s[idx:idx + 3] == "NaN":
                idx, mode = idx + 3, "after"
            elif c == "I" and s[idx:idx + 8] == "Infinity":
                idx, mode = idx + 8, "after"
            elif c == "-" and s[idx:idx + 9] == "-Infinity":
                idx, mode = idx + 9, "after"
            else:
                end = _number(s, idx)
                if end is None:
                    raise _Decided(True)       # Expecting value
                idx, mode = end, "after"
        elif mode == "key":
            if idx >= n or s[idx] != '"':
                raise _Decided(True)           # Expecting property name enclosed in double quotes
            idx = _skip_ws(s, _scanstring(s, idx + 1))
            if idx >= n or s[idx] != ":":
                raise _Decided(True)           # Expecting ':' delimiter
            idx = _skip_ws(s, idx + 1)
            mode = "value"
        else:  # after a value
            if not stack:
                return idx
            idx = _skip_ws(s, idx)
            top = stack[-1]
            if idx < n and s[idx] == ("}" if top == "{" else "]"):
                stack.pop()
                idx += 1
                continue
            if idx >= n or s[idx] != ",":
                raise _Decided(True)           # Expecting ',' delimiter
            idx = _skip_ws(s, idx + 1)
            mode = "key" if top == "{" else "value"


def is_valid_prefix(s: str) -> Answer:
    """The reference's answer for `s`: True, False, or RAISE."""
    if not s or s.startswith("{"):
        return True
    try:
        end = _skip_ws(s, _scan(s))
    except _Decided as d:
        return d.ok
    except _Raises:
        return RAISE
    return end == len(s)                       # else "Extra data"


def token_mask(prefix: str, vocab: List[str]) -> List[Answer]:
    """allowed[t] for every token of the vocabulary."""
    return [is_valid_prefix(prefix + t) for t in vocab]


def pack_mask(answers: List[Answer]):
    """[ceil(V/32)] uint32 words, bit (t & 31) of word (t >> 5) = allowed."""
    import numpy as np
    V = len(answers)
    bits = np.zeros(((V + 31) // 32) * 32, np.uint8)
    bits[:V] = [1 if a is True else 0 for a in answers]
    return np.packbits(bits.reshape(-1, 32)[:, ::-1], axis=1, bitorder="big").view(">u4").astype(np.uint32).ravel()
