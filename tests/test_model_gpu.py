"""GPU parity of the Qwen3-4B-shaped decode runtime
against the CPU oracle model, through the C ABI.

The runtime follows the oracle's operation order everywhere, so the bar is
bit-identical logits at every step (which implies identical greedy tokens).
The reference's own integration check compares full-vocabulary logit dumps
step by step (tests/runtime_logits.cpp:59-108, tools/compare-runtime-logits.py)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _pair(**cfg):
    from abra_b200.model import DecodeModel

    return DecodeModel(**cfg), O.OrcModel(**cfg)


def _prompt(n, vocab, seed):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


@pytest.mark.parametrize("centered", [1, 0])
def test_small_model_logits_bit_exact_across_chunks(centered):
    """2 layers, vocab 4096, 600 positions: attention crosses the 256-position
    chunk boundaries; logits compared at every step of a window around each."""
    cfg = dict(n_layers=2, vocab=4096, max_ctx=600, centered=centered, seed=3)
    g, c = _pair(**cfg)
    prompt = _prompt(5, 4096, 1)
    g.reset(prompt)
    check = set(range(0, 12)) | set(range(250, 262)) | set(range(508, 516)) | {598}
    tok = None
    for pos in range(599):
        feed = int(prompt[pos]) if pos < len(prompt) else tok
        want_tok, want = c.step(feed, pos, logits=True)
        g.step(1)
        if pos in check:
            got = g.logits()
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"logits differ at pos {pos}"
        tok = want_tok
    toks = g.tokens(600)
    assert g.position() == 599
    assert np.array_equal(toks[:5], prompt)
    g.close()
    c.close()


def test_persistent_kernel_is_the_default_step():
    """Batch 1 on one GPU with all-Q4_K weights runs the persistent decode
    kernel; the flag selects the kernel chain; the Q4_K_M map keeps the chain."""
    from abra_b200.model import KERNEL_CHAIN, Q4_K_M, DecodeModel

    cfg = dict(n_layers=1, vocab=512, max_ctx=8)
    with DecodeModel(**cfg) as m:
        assert m.persistent
    with DecodeModel(flags=KERNEL_CHAIN, **cfg) as m:
        assert not m.persistent
    with DecodeModel(flags=Q4_K_M, **cfg) as m:
        assert not m.persistent


@pytest.mark.parametrize("shape", [
    dict(hidden=512, n_heads=4, n_kv_heads=2, ffn=1024),   # 2 q heads per kv head
    dict(hidden=512, n_heads=8, n_kv_heads=1, ffn=768),    # 8
    dict(hidden=256, n_heads=2, n_kv_heads=2, ffn=512),    # 1, one superblock per row
])
def test_persistent_gqa_shapes_bit_exact_across_chunks(shape):
    """The persistent kernel's attention items, per-group merge counters and
    GEMV plans on other head layouts and widths: logits bit-identical to the
    oracle around each 256-position chunk boundary."""
    from abra_b200.model import DecodeModel

    cfg = dict(n_layers=2, vocab=1000, max_ctx=530, centered=1, seed=4, **shape)
    g, c = DecodeModel(**cfg), O.OrcModel(**cfg)
    assert g.persistent
    prompt = _prompt(3, 1000, 5)
    g.reset(prompt)
    check = {0, 1, 2, 254, 255, 256, 257, 511, 512, 513, 528}
    tok, picks = None, []
    for pos in range(529):
        feed = int(prompt[pos]) if pos < len(prompt) else tok
        want_tok, want = c.step(feed, pos, logits=True)
        g.step(1)
        if pos in check:
            got = g.logits()
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"logits differ at pos {pos}"
        tok = want_tok
        if pos >= 2:
            picks.append(tok)
    assert np.array_equal(g.tokens(530)[3:], np.array(picks, dtype=np.int32))
    g.close()
    c.close()


def test_persistent_eight_slot_ring_bit_exact():
    """A 4096-wide model with a 14336-wide FFN: its activations leave shared
    memory for eight ring slots only, so each warp refills the slot it
    finished with the unit eight tickets ahead.  Logits bit-identical to the
    oracle at every step."""
    from abra_b200.model import DecodeModel, persist_plan

    shape = dict(hidden=4096, n_heads=32, n_kv_heads=8, ffn=14336)
    assert persist_plan(148, n_layers=2, vocab=1000, **shape)["ring_bytes"] == 8 * 8 * 1456
    cfg = dict(n_layers=2, vocab=1000, max_ctx=64, centered=1, seed=6, **shape)
    g, c = DecodeModel(**cfg), O.OrcModel(**cfg)
    assert g.persistent
    prompt = _prompt(3, 1000, 7)
    g.reset(prompt)
    tok = None
    for pos in range(24):
        feed = int(prompt[pos]) if pos < len(prompt) else tok
        tok, want = c.step(feed, pos, logits=True)
        g.step(1)
        got = g.logits()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"logits differ at pos {pos}"
    g.close()
    c.close()


def test_graph_eager_no_pdl_and_no_prefetch_agree():
    """Every way of running the step -- the persistent kernel as a graph or
    eager, the kernel chain with and without graphs, PDL and L2 prefetch --
    gives the same tokens and logit bits."""
    from abra_b200.model import EAGER, KERNEL_CHAIN, NO_PDL, NO_PREFETCH, DecodeModel

    cfg = dict(n_layers=3, vocab=2048, max_ctx=300, centered=1, seed=5)
    prompt = _prompt(7, 2048, 2)
    outs = []
    for flags in (0, EAGER, KERNEL_CHAIN, KERNEL_CHAIN | EAGER, KERNEL_CHAIN | NO_PDL,
                  KERNEL_CHAIN | EAGER | NO_PDL, KERNEL_CHAIN | NO_PREFETCH):
        with DecodeModel(flags=flags, **cfg) as m:
            toks = m.generate(prompt, 280)
            outs.append((toks, m.logits()))
    for toks, lg in outs[1:]:
        assert np.array_equal(toks, outs[0][0])
        assert np.array_equal(lg.view(np.uint32), outs[0][1].view(np.uint32))


def test_streaming_loop_matches_graph_replay():
    from abra_b200.model import DecodeModel

    cfg = dict(n_layers=2, vocab=3000, max_ctx=80, centered=1, seed=11)
    prompt = _prompt(9, 3000, 4)
    with DecodeModel(**cfg) as a, DecodeModel(**cfg) as b:
        want = a.generate(prompt, 40)
        b.reset(prompt)
        b.step(len(prompt) - 1)
        got = b.decode_streaming(40)
        assert np.array_equal(got, want)
        assert b.position() == len(prompt) - 1 + 40
        with pytest.raises(Exception):
            b.step(80)  # would pass max_ctx: refused on the host


@pytest.mark.parametrize("centered", [1, 0])
def test_full_qwen3_4b_shape_greedy_bit_exact(centered):
    """The full 36-layer Qwen3-4B shape, 16-token prompt, 16 greedy steps:
    logits bit-identical to the CPU oracle at every step."""
    cfg = dict(max_ctx=64, centered=centered, seed=0)
    g, c = _pair(**cfg)
    prompt = _prompt(16, 151936, 7)
    g.reset(prompt)
    tok = None
    picks = []
    for pos in range(32):
        feed = int(prompt[pos]) if pos < 16 else tok
        tok, want = c.step(feed, pos, logits=True)
        g.step(1)
        got = g.logits()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"pos {pos}"
        if pos >= 15:
            picks.append(tok)
    assert np.array_equal(g.tokens(33)[16:33], np.array(picks, dtype=np.int32))
    if centered:
        assert len(set(picks)) > 4, "centred model should not collapse to one token"
    g.close()
    c.close()


def test_full_qwen3_4b_tg128_greedy_tokens_identical():
    """The decode bar at the benchmark's length: the full 36-layer shape, a
    16-token prompt, tg128 -- the 128 greedy token ids equal the CPU oracle's,
    and the logits of the last step are bit-identical."""
    cfg = dict(max_ctx=160, centered=1, seed=0)
    g, c = _pair(**cfg)
    prompt = _prompt(16, 151936, 9)
    got = g.generate(prompt, 128)
    last = g.logits()
    want, tok = [], None
    for pos in range(16 + 127):
        feed = int(prompt[pos]) if pos < 16 else tok
        if pos == 16 + 126:
            tok, want_logits = c.step(feed, pos, logits=True)
        else:
            tok = c.step(feed, pos)
        if pos >= 15:
            want.append(tok)
    want = np.array(want, dtype=np.int32)
    bad = np.flatnonzero(got != want)
    assert bad.size == 0, f"tokens first differ at step {bad[:1]}: {got[bad[:4]]} vs {want[bad[:4]]}"
    assert np.array_equal(last.view(np.uint32), want_logits.view(np.uint32))
    assert len(set(want.tolist())) > 8, "the centred model should not collapse to a few tokens"
    g.close()
    c.close()


def _mix_pair(**cfg):
    from abra_b200.model import Q4_K_M, DecodeModel

    return DecodeModel(flags=Q4_K_M, **cfg), O.OrcModel(mix=1, **cfg)


def test_q4_k_m_type_map_small_model_bit_exact():
    """9 layers under the Q4_K_M type map (Q6_K attn_v/ffn_down in layers 0,
    3, 6, 7, 8, Q6_K tied table): logits bit-identical to the oracle."""
    cfg = dict(n_layers=9, vocab=4096, max_ctx=300, centered=1, seed=13)
    g, c = _mix_pair(**cfg)
    prompt = _prompt(6, 4096, 5)
    g.reset(prompt)
    tok = None
    for pos in range(40):
        feed = int(prompt[pos]) if pos < len(prompt) else tok
        tok, want = c.step(feed, pos, logits=True)
        g.step(1)
        got = g.logits()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"logits differ at pos {pos}"
    g.close()
    c.close()


def test_q4_k_m_graph_eager_no_pdl_no_prefetch_agree():
    from abra_b200.model import EAGER, NO_PDL, NO_PREFETCH, Q4_K_M, DecodeModel

    cfg = dict(n_layers=5, vocab=2048, max_ctx=200, centered=1, seed=17)
    prompt = _prompt(4, 2048, 6)
    outs = []
    for flags in (0, EAGER, NO_PDL, NO_PREFETCH):
        with DecodeModel(flags=flags | Q4_K_M, **cfg) as m:
            outs.append((m.generate(prompt, 150), m.logits()))
    for toks, lg in outs[1:]:
        assert np.array_equal(toks, outs[0][0])
        assert np.array_equal(lg.view(np.uint32), outs[0][1].view(np.uint32))


def test_full_qwen3_4b_q4_k_m_greedy_bit_exact():
    """The full 36-layer shape with the real Q4_K_M type map (18 Q6_K layers,
    Q6_K tied 151936 x 2560 table): logits bit-identical at every step."""
    cfg = dict(max_ctx=64, centered=1, seed=0)
    g, c = _mix_pair(**cfg)
    prompt = _prompt(16, 151936, 8)
    g.reset(prompt)
    tok = None
    for pos in range(24):
        feed = int(prompt[pos]) if pos < 16 else tok
        tok, want = c.step(feed, pos, logits=True)
        g.step(1)
        assert np.array_equal(g.logits().view(np.uint32), want.view(np.uint32)), f"pos {pos}"
    g.close()
    c.close()


def test_prefill_matches_token_by_token_decode():
    """Prompt processing on the tensor cores leaves the KV cache bit-identical
    to decoding the prompt token by token: the logits of every following step
    are equal (2 layers; 300 prompt tokens cross a 256-position attention
    chunk; chunks of 256 + 32, then a second prefill from a later position)."""
    from abra_b200.model import DecodeModel

    cfg = dict(n_layers=2, vocab=4096, max_ctx=400, centered=1, seed=21)
    prompt = _prompt(330, 4096, 9)
    with DecodeModel(**cfg) as a, DecodeModel(**cfg) as b:
        a.reset(prompt)
        b.reset(prompt)
        b.step(5)
        b.prefill(288)    # positions 5..292: one 256 chunk and one 32 chunk
        b.prefill(32)     # positions 293..324
        a.step(325)
        assert b.position() == a.position() == 325
        for pos in range(325, 340):
            a.step(1)
            b.step(1)
            assert np.array_equal(a.logits().view(np.uint32), b.logits().view(np.uint32)), f"pos {pos}"
        assert np.array_equal(a.tokens(341), b.tokens(341))


def test_prefill_full_shape_matches_decode_and_refuses_bad_calls():
    from abra_b200.model import DecodeModel, Q4_K_M
    from abra_b200._lib import AbraError

    cfg = dict(max_ctx=160, centered=1, seed=2)
    prompt = _prompt(129, 151936, 10)
    with DecodeModel(**cfg) as a, DecodeModel(**cfg) as b:
        a.feed_prompt(prompt)   # prefill 128, then the last prompt token
        b.reset(prompt)
        b.step(129)
        for pos in range(129, 137):
            assert np.array_equal(a.logits().view(np.uint32), b.logits().view(np.uint32)), f"pos {pos}"
            a.step(1)
            b.step(1)
        with pytest.raises(Exception):
            a.prefill(32)  # past the prompt
    with DecodeModel(max_ctx=64, n_layers=2, vocab=512, flags=Q4_K_M) as m:
        m.reset(_prompt(40, 512, 1))
        with pytest.raises(AbraError):
            m.prefill(32)  # the Q4_K_M map has no tensor-core path


# (vocab, centered, seed, proposed, accepted): with the 64-token vocabulary the
# greedy output cycles, so drafts are proposed, partly accepted and partly
# rejected -- the counts follow from the greedy tokens by the reference's
# draft rule (the CPU oracle's tokens, which the GPU reproduces bit for bit);
# the all-4096 non-centred model repeats one token, which never drafts.
LOOKUP_CASES = [(4096, 0, 31, 0, 0), (64, 1, 5, 236, 32)]


@pytest.mark.parametrize("vocab,centered,seed,proposed,accepted", LOOKUP_CASES)
def test_lookup_decoding_equals_greedy(vocab, centered, seed, proposed, accepted):
    """Prompt-lookup speculation (drafts verified in 32-column passes) gives
    exactly the greedy tokens, with the draft counts of the reference's rule."""
    from abra_b200.model import DecodeModel

    cfg = dict(n_layers=2, vocab=vocab, max_ctx=400, centered=centered, seed=seed)
    base = _prompt(20, vocab, 12)
    prompt = np.concatenate([base, base[:12], base]).astype(np.int32)  # repeats to look up
    with DecodeModel(**cfg) as m:
        want = m.generate(prompt, 120)
        got, stats = m.generate_lookup(prompt, 120, key=2, draft_max=16)
        assert np.array_equal(got, want)
        assert (stats["proposed"], stats["accepted"]) == (proposed, accepted), stats
        # the state after lookup decoding continues like greedy decoding
        m.step(1)
        after = m.tokens(len(prompt) + 121)[len(prompt) + 120]
    with DecodeModel(**cfg) as g:
        assert g.generate(prompt, 121)[120] == after


def test_verify_picks_are_the_decode_steps_picks():
    from abra_b200.model import DecodeModel

    cfg = dict(n_layers=2, vocab=4096, max_ctx=200, centered=1, seed=33)
    prompt = _prompt(9, 4096, 13)
    with DecodeModel(**cfg) as a, DecodeModel(**cfg) as b:
        greedy = a.generate(prompt, 20)
        b.reset(prompt)
        b.step(9)                   # current = greedy[0] at position 9
        draft = np.array(list(greedy[1:6]) + [7, 8], dtype=np.int32)  # 5 right, then wrong
        kept, picks = b.verify(draft)
        assert kept == 6 and np.array_equal(picks[:6], greedy[1:7])
        assert b.position() == 15
        b.step(4)
        assert np.array_equal(b.tokens(20)[9:20], greedy[:11])
