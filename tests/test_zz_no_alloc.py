"""ms_build_json_mask_noalloc: the JSON-grammar mask build for callers that
cannot allocate device memory (a serving runtime that hands out all device
memory from its own pool, or a plugin with no device allocator it may call).
Its vocabulary tables live in a fixed device array inside the library; the
masks and statuses must equal those of the existing entry point, which reads
the same tables from caller memory (ms_build_json_mask_packed), on two calls
in a row with different vocabularies and states.  This file is collected
last so that a run stopping at the first failure has run every other test.
Needs a B200."""
import random

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    if not t.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return t


def _vocab(seed, n):
    from miniserve_b200 import workloads
    vocab = workloads.json_vocab(seed, n)
    rng = random.Random(seed)
    for i in range(0, len(vocab), 89):  # some tokens longer than 16 bytes
        vocab[i] = "".join(rng.choice('{}[]:," 0123456789.eE-truefalsn\\') for _ in range(rng.randint(17, 40)))
    return vocab


def test_noalloc_mask_matches_packed_entry_point(torch):
    from miniserve_b200 import _lib, workloads
    from miniserve_b200.grammar import JsonMaskBuilder
    L = _lib.lib()
    sp = torch.cuda.current_stream().cuda_stream
    # two calls in a row: the second with a smaller vocabulary and other states,
    # so nothing of the first call's tables may show through
    for seed, nvocab, nrows in ((4, 20011, 64), (5, 9000, 40)):
        b = JsonMaskBuilder(_vocab(seed, nvocab), order=None)
        prefixes = workloads.json_prefixes(seed, nrows) + ["[1, 2", '{"a": "x', ""]
        s = b.init(prefixes)
        want_mask, want_st = b.build(s, packed=True)  # the existing entry point, caller-owned tables
        B, V = len(prefixes), nvocab
        W = (V + 31) // 32
        mask = torch.full((B, W), -1, dtype=torch.int32, device="cuda")
        st = torch.full((B,), -7, dtype=torch.int32, device="cuda")
        _lib.check(L.ms_build_json_mask_noalloc(s.data_ptr(), B, b.vocab_bytes.data_ptr(), b.vocab_off.data_ptr(),
                                                V, mask.data_ptr(), W, st.data_ptr(), sp),
                   "ms_build_json_mask_noalloc")
        torch.cuda.synchronize()
        np.testing.assert_array_equal(mask.cpu().numpy(), want_mask.cpu().numpy())
        np.testing.assert_array_equal(st.cpu().numpy(), want_st.cpu().numpy())


def test_noalloc_rejects_vocabulary_beyond_its_array(torch):
    from miniserve_b200 import _lib
    L = _lib.lib()
    V = 262145
    W = (V + 31) // 32
    mask = torch.empty((1, W), dtype=torch.int32, device="cuda")
    st = torch.empty(1, dtype=torch.int32, device="cuda")
    states = torch.zeros((1, 64), dtype=torch.int32, device="cuda")
    vb = torch.zeros(16, dtype=torch.uint8, device="cuda")
    vo = torch.zeros(V + 1, dtype=torch.int64, device="cuda")
    rc = L.ms_build_json_mask_noalloc(states.data_ptr(), 1, vb.data_ptr(), vo.data_ptr(), V, mask.data_ptr(), W,
                                      st.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.MS_E_TOO_LARGE
    assert "262144" in L.ms_error_string(rc).decode()
