"""The GPU JSON-grammar mask against the oracle (oracle/json_prefix.py, pinned
to miniserve's is_valid_prefix) and the reference's golden answers; then the
masked sampling of config 4 against the C oracle.  Needs a B200."""
import json
import os
import random

import numpy as np
import pytest

from oracle import json_prefix as jp
from parity import compare

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    if not t.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return t


def _bits(mask_row, V):
    w = np.asarray(mask_row).view(np.uint32)
    return ((w[:, None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(-1)[:V].astype(bool)


def test_golden_strings_split_at_every_point(torch):
    """Each golden string, split into (prefix, token) at several points, gives
    the reference's answer (a raise gives bit 0 and row status 1)."""
    from miniserve_b200.grammar import JsonMaskBuilder
    with open(os.path.join(HERE, "golden", "json_prefix_golden.json")) as f:
        cases = json.load(f)["cases"]
    rng = random.Random(5)
    pairs = []
    for s, a in cases:
        for k in sorted({0, len(s), rng.randint(0, len(s))}):
            pairs.append((s[:k], s[k:], a))
    # one row per distinct prefix, the tokens as the vocabulary
    tokens = sorted({t for _, t, _ in pairs})
    tid = {t: i for i, t in enumerate(tokens)}
    prefixes = sorted({p for p, _, _ in pairs})
    pid = {p: i for i, p in enumerate(prefixes)}
    b = JsonMaskBuilder(tokens)
    bad = []
    for lo in range(0, len(prefixes), 4096):
        chunk = prefixes[lo:lo + 4096]
        mask, st = b.build(b.init(chunk))
        torch.cuda.synchronize()
        m = mask.cpu().numpy()
        for p, t, a in pairs:
            i = pid[p] - lo
            if 0 <= i < len(chunk):
                got = bool(_bits(m[i], len(tokens))[tid[t]])
                if got != (a is True):
                    bad.append((p, t, a))
    assert not bad, bad[:10]


def test_config4_masks_vs_oracle(torch):
    """Config-4 rows: full-vocabulary masks for the short prefixes, sampled
    tokens for the long ones."""
    from miniserve_b200 import workloads
    from miniserve_b200.grammar import JsonMaskBuilder
    V = 151936
    vocab = workloads.json_vocab(4, V)
    prefixes = workloads.json_prefixes(4, 128)
    b = JsonMaskBuilder(vocab)
    mask, st = b.build(b.init(prefixes))
    torch.cuda.synchronize()
    m = mask.cpu().numpy()
    assert not st.cpu().numpy().any()
    rng = random.Random(11)
    checked = 0
    full_rows = 0
    for r, p in enumerate(prefixes):
        bits = _bits(m[r], V)
        if len(p) <= 8 and full_rows < 12:
            full_rows += 1
            idx = range(V)
        else:
            idx = rng.sample(range(V), 300 if len(p) < 2000 else 40)
        for t in idx:
            want = jp.is_valid_prefix(p + vocab[t]) is True
            assert bits[t] == want, (r, p[-30:], vocab[t], want)
            checked += 1
    assert checked > 10 * V


def test_masks_match_reference_fuzz_fixture(torch):
    """Miniserve's own answers for 10^6 (state, token) pairs
    (tests/golden/json_mask_fuzz.npz: 40 parse states over the 151936-token
    config-4 vocabulary): the GPU mask bit of every pair, in the default
    (length-ordered) and token-ordered builds."""
    import golden_util
    from miniserve_b200 import workloads
    from miniserve_b200.grammar import JsonMaskBuilder
    prefixes, tokens, allowed, raises = golden_util.load_mask_fuzz()
    vocab = workloads.json_vocab(4)
    for order in ("length", None):
        b = JsonMaskBuilder(vocab, order=order)
        mask, st = b.build(b.init(prefixes))
        torch.cuda.synchronize()
        m = mask.cpu().numpy().view(np.uint32)
        got = ((m[np.arange(len(prefixes))[:, None], tokens >> 5] >> (tokens & 31).astype(np.uint32)) & 1).astype(bool)
        want = allowed.copy()
        for i, j in raises:  # a raise: bit 0 and row status 1
            want[i, j] = False
            assert st.cpu().numpy()[i] & 1
        if not raises:
            assert not st.cpu().numpy().any()
        bad = np.argwhere(got != want)
        assert len(bad) == 0, [(prefixes[i][-30:], vocab[tokens[i, j]], bool(want[i, j])) for i, j in bad[:10]]
    assert tokens.size == 1_000_000


def test_advance_matches_init(torch):
    """State after prefix + sampled token == state built from the joined text."""
    from miniserve_b200 import workloads
    from miniserve_b200.grammar import JsonMaskBuilder
    vocab = workloads.json_vocab(4, 4096)
    prefixes = [p for p in workloads.json_prefixes(4, 128) if len(p) < 600][:48]
    b = JsonMaskBuilder(vocab)
    rng = np.random.default_rng(2)
    toks = rng.integers(0, len(vocab), len(prefixes))
    s1 = b.init(prefixes)
    b.advance(s1, torch.from_numpy(toks))
    s2 = b.init([p + vocab[t] for p, t in zip(prefixes, toks)])
    m1, _ = b.build(s1)
    m2, _ = b.build(s2)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(m1.cpu().numpy(), m2.cpu().numpy())


def test_rows_in_one_state_share_a_mask(torch):
    """Rows in the same parse state share one mask computation (a dedup pass);
    rows whose states differ only in the container stack, or only in deep
    levels of it, keep their own masks.  Every row equals its single-row
    build."""
    from miniserve_b200 import workloads
    from miniserve_b200.grammar import JsonMaskBuilder
    vocab = workloads.json_vocab(4, 12000)
    base = ['{"a": [1, "x', '{"a": {"b": "x', '[[[[{"k": [', '[[{[{"k": [', '[{[[{"k": [', "[1, 2", "[1, 2",
            '{"a": [1, "x', "", "tru", '"\\u00', "[" * 40 + "{" + '"k": ', "[" * 39 + "{[" + '"k": ']
    prefixes = [base[i % len(base)] for i in range(3 * len(base))]
    b = JsonMaskBuilder(vocab)
    m, st = b.build(b.init(prefixes))
    torch.cuda.synchronize()
    m = m.cpu().numpy()
    st = st.cpu().numpy()
    for i, p in enumerate(prefixes[:len(base)]):
        m1, st1 = b.build(b.init([p]))
        torch.cuda.synchronize()
        for j in range(i, len(prefixes), len(base)):
            np.testing.assert_array_equal(m[j], m1.cpu().numpy()[0], err_msg=repr(p))
            assert st[j] == st1.cpu().numpy()[0]


def test_packed_matches_unpacked(torch):
    """The fixed-width vocabulary path gives the same masks and statuses as the
    variable-length one, tokens longer than 16 bytes included."""
    from miniserve_b200 import workloads
    from miniserve_b200.grammar import JsonMaskBuilder
    vocab = workloads.json_vocab(4, 20000)
    rng = random.Random(3)
    for i in range(0, len(vocab), 97):  # some long tokens (17-40 bytes)
        vocab[i] = "".join(rng.choice('{}[]:," 0123456789.eE-truefalsn\\') for _ in range(rng.randint(17, 40)))
    prefixes = workloads.json_prefixes(4, 96)
    b = JsonMaskBuilder(vocab)
    s = b.init(prefixes)
    m1, st1 = b.build(s, packed=True)
    m2, st2 = b.build(s, packed=False)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(m1.cpu().numpy(), m2.cpu().numpy())
    np.testing.assert_array_equal(st1.cpu().numpy(), st2.cpu().numpy())
    lens = b.lens.cpu().numpy()
    assert (lens == 255).sum() == sum(len(v.encode()) > 16 for v in vocab)


def test_config4_masked_sampling(torch):
    """Config 4 end to end: masks on the GPU, masked sampling vs the C oracle
    with the same mask."""
    from miniserve_b200 import Sampler, workloads
    from miniserve_b200.grammar import JsonMaskBuilder
    cfg = workloads.config4(4, B=128)
    b = JsonMaskBuilder(cfg.extra["vocab"])
    mask, st = b.build(b.init(cfg.extra["prefixes"]))
    x = torch.from_numpy(cfg.logits).cuda()
    tok, prob, status = Sampler().sample_batch(x, cfg.temperature, cfg.top_k, cfg.top_p, uniforms=cfg.uniforms,
                                               mask=mask)
    torch.cuda.synchronize()
    compare(tok.cpu().numpy(), prob.cpu().numpy().astype(np.float64), status.cpu().numpy(), cfg.logits,
            cfg.temperature, cfg.top_k, cfg.top_p, cfg.uniforms, mask=mask.cpu().numpy().view(np.uint32),
            label="config4 masked")


def test_ordered_matches_token_order(torch):
    """The length-ordered vocabulary path gives the same masks and statuses as
    token order: long tokens, a vocabulary that is not a multiple of 32, rows
    that share a state, and an arbitrary permutation through the C ABI."""
    from miniserve_b200 import _lib, workloads
    from miniserve_b200.grammar import JsonMaskBuilder
    vocab = workloads.json_vocab(4, 20011)
    rng = random.Random(7)
    for i in range(0, len(vocab), 89):  # some long tokens (17-40 bytes)
        vocab[i] = "".join(rng.choice('{}[]:," 0123456789.eE-truefalsn\\') for _ in range(rng.randint(17, 40)))
    prefixes = workloads.json_prefixes(4, 64)
    prefixes = prefixes + prefixes[:20] + ["[1, 2", "[1, 2", '{"a": "x', ""]
    ordered = JsonMaskBuilder(vocab)
    plain = JsonMaskBuilder(vocab, order=None)
    assert ordered.order is not None and plain.order is None
    s = ordered.init(prefixes)
    m1, st1 = ordered.build(s)
    m2, st2 = plain.build(s)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(m1.cpu().numpy(), m2.cpu().numpy())
    np.testing.assert_array_equal(st1.cpu().numpy(), st2.cpu().numpy())
    assert sorted(ordered.order.cpu().tolist()) == list(range(len(vocab)))
    # any permutation gives the same masks; a padded row stride too
    V = len(vocab)
    perm = torch.from_numpy(np.random.default_rng(3).permutation(V).astype(np.int32)).cuda()
    packed = torch.empty((V, 4), dtype=torch.int32, device="cuda")
    lens = torch.empty(V, dtype=torch.uint8, device="cuda")
    L = _lib.lib()
    sp = torch.cuda.current_stream().cuda_stream
    _lib.check(L.ms_json_pack_vocab_ordered(ordered.vocab_bytes.data_ptr(), ordered.vocab_off.data_ptr(), V,
                                            perm.data_ptr(), packed.data_ptr(), lens.data_ptr(), sp),
               "ms_json_pack_vocab_ordered")
    B = len(prefixes)
    W = (V + 31) // 32
    m3 = torch.full((B, W + 5), -1, dtype=torch.int32, device="cuda")
    st3 = torch.empty(B, dtype=torch.int32, device="cuda")
    _lib.check(L.ms_build_json_mask_ordered(s.data_ptr(), B, ordered.vocab_bytes.data_ptr(),
                                            ordered.vocab_off.data_ptr(), packed.data_ptr(), lens.data_ptr(),
                                            perm.data_ptr(), V, m3.data_ptr(), W + 5,
                                            st3.data_ptr(), sp), "ms_build_json_mask_ordered")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(m3[:, :W].cpu().numpy(), m2.cpu().numpy())
    assert (m3[:, W:].cpu().numpy() == -1).all()  # the padding is untouched
    np.testing.assert_array_equal(st3.cpu().numpy(), st2.cpu().numpy())
    # the ordered path refuses a missing order
    assert L.ms_build_json_mask_ordered(s.data_ptr(), B, ordered.vocab_bytes.data_ptr(),
                                        ordered.vocab_off.data_ptr(), packed.data_ptr(), lens.data_ptr(),
                                        None, V, m3.data_ptr(), W + 5, st3.data_ptr(), sp) != 0
