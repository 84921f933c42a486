"""Inference stack on CPU (fp32): KV-cache decode vs full recomputation, reference parity
of the decoders, sampling filters, streaming, chat sessions, speculative decoding, Engram."""

import pytest
import torch

from saint_llm_b200.config import ModelConfig
from saint_llm_b200.data import CharTokenizer, ChatTemplate, ChatTurn
from saint_llm_b200.infer import (
    ChatSession,
    EAGLE3Config,
    EAGLE3DraftHead,
    EngramConfig,
    EngramHook,
    EngramTable,
    GenerationConfig,
    KVCacheBundle,
    StopSequenceMatcher,
    apply_logit_bias,
    build_multimodal_prompt_ids,
    forbid_tokens_bias,
    greedy_decode,
    greedy_decode_cached,
    speculative_decode,
    stream_greedy_decode,
    stream_top_p_sample,
    top_k_sample,
    top_k_sample_cached,
    top_p_sample,
    top_p_sample_cached,
)
from saint_llm_b200.infer.engram import ngram_buckets, trailing_bucket
from saint_llm_b200.infer.sampling import filter_top_p
from saint_llm_b200.models import SaintLLM


def _model(update=None):
    cfg = ModelConfig.tiny()
    if update:
        cfg = cfg.model_copy(update=update)
    torch.manual_seed(0)
    return SaintLLM(cfg).eval()


@pytest.fixture(scope="module")
def model():
    return _model()


def _prompt(b=2, t=13, vocab=512, seed=1):
    return torch.randint(0, vocab, (b, t), generator=torch.Generator().manual_seed(seed))


def test_cached_logits_match_full_forward(model):
    ids = _prompt(t=21)
    full = model(ids)["logits"]
    bundle = KVCacheBundle.for_model(model, max_seq_len=40, batch_size=2)
    chunks = [ids[:, :9], ids[:, 9:10], ids[:, 10:17], ids[:, 17:18], ids[:, 18:21]]
    got = torch.cat([model(c, kv_cache_bundle=bundle)["logits"] for c in chunks], dim=1)
    assert bundle.length == 21
    torch.testing.assert_close(got, full, rtol=1e-4, atol=1e-4)


def test_greedy_cached_equals_uncached(model):
    ids = _prompt()
    a = greedy_decode(model, ids, max_new_tokens=12)
    b = greedy_decode_cached(model, ids, max_new_tokens=12)
    assert a.shape == (2, 25)
    assert torch.equal(a, b)


def test_eos_padding_contract(model):
    ids = _prompt()
    free = greedy_decode(model, ids, max_new_tokens=10)
    eos = int(free[0, ids.shape[1] + 1])  # row 0's second generated token
    out = greedy_decode_cached(model, ids, max_new_tokens=10, eos_token=eos)
    assert out.shape == free.shape
    seen = (out[:, ids.shape[1]:] == eos).cumsum(1) > 0
    all_done = seen.all(0)
    if bool(all_done.any()):
        first = int(all_done.nonzero()[0])
        assert bool((out[:, ids.shape[1] + first + 1:] == eos).all())


def test_decoders_match_reference(ref_pkgs, model):
    from saint_llm_core.config import ModelConfig as RC
    from saint_llm_core.model import SaintLLM as RM
    from saint_llm_inference import generate as rg

    torch.manual_seed(0)
    ref = RM(RC.tiny()).eval()
    ref.load_state_dict(model.state_dict())
    ids = _prompt()
    assert torch.equal(greedy_decode(model, ids, max_new_tokens=8), rg.greedy_decode(ref, ids, max_new_tokens=8))
    for ours, theirs, kw in [
        (top_k_sample, rg.top_k_sample, {"k": 20, "temperature": 0.8, "repetition_penalty": 1.3}),
        (top_p_sample, rg.top_p_sample, {"p": 0.8, "temperature": 0.9, "top_k": 64}),
    ]:
        a = ours(model, ids, max_new_tokens=6, generator=torch.Generator().manual_seed(5), **kw)
        b = theirs(ref, ids, max_new_tokens=6, generator=torch.Generator().manual_seed(5), **kw)
        assert torch.equal(a, b), ours.__name__


def test_cached_samplers_equal_uncached(model):
    ids = _prompt()
    for f, g, kw in [(top_k_sample, top_k_sample_cached, {"k": 10}), (top_p_sample, top_p_sample_cached, {"p": 0.7})]:
        a = f(model, ids, max_new_tokens=7, generator=torch.Generator().manual_seed(3), **kw)
        b = g(model, ids, max_new_tokens=7, generator=torch.Generator().manual_seed(3), **kw)
        assert torch.equal(a, b)


def test_top_p_filter_keeps_best_and_minimal_prefix():
    logits = torch.log(torch.tensor([[0.5, 0.3, 0.15, 0.05]]))
    out = filter_top_p(logits, 0.7)
    assert torch.isfinite(out).tolist() == [[True, True, False, False]]
    assert torch.isfinite(filter_top_p(logits, 1e-6)).sum() == 1


def test_logit_bias_and_stop_matcher():
    x = torch.zeros(2, 8)
    y = apply_logit_bias(x, {3: 2.0, 100: 5.0, **forbid_tokens_bias([1])})
    assert y[0, 3] == 2.0 and y[1, 1] == -1e9 and y.sum() == 2 * (2.0 - 1e9)
    m = StopSequenceMatcher([[10, 11], [20], []])
    assert [m.feed(t) for t in (7, 10, 11, 5)] == [False, False, True, True]
    assert m.matched_sequence == (10, 11)


def test_streaming_matches_greedy_and_stops(model):
    ids = _prompt(b=1)
    full = greedy_decode(model, ids, max_new_tokens=6)
    got = torch.cat(list(stream_greedy_decode(model, ids, max_new_tokens=6)), dim=1)
    assert torch.equal(got, full[:, ids.shape[1]:])
    stop = [int(full[0, ids.shape[1] + 1]), int(full[0, ids.shape[1] + 2])]
    got = list(stream_greedy_decode(model, ids, max_new_tokens=6, stop_sequences=[stop], use_cache=False))
    m = StopSequenceMatcher([stop])
    expect = next(i + 1 for i, t in enumerate(full[0, ids.shape[1]:].tolist()) if m.feed(t))
    assert len(got) == expect
    s = list(stream_top_p_sample(model, ids, max_new_tokens=4, temperature=0.0))
    assert torch.equal(torch.cat(s, 1), full[:, ids.shape[1]:ids.shape[1] + 4])


def test_chat_session_roundtrip(model):
    tok = CharTokenizer(base_vocab=16, unicode_max=512 - 16)
    sess = ChatSession(model=model, tokenizer=tok, system="be brief", template=ChatTemplate(
        system_prefix="S:", system_suffix="\n", user_prefix="U:", user_suffix="\n", assistant_prefix="A:",
        assistant_suffix="\n"))
    sess.add_user("hi")
    text = sess.respond(cfg=GenerationConfig(max_new_tokens=5, temperature=0.0))
    assert isinstance(text, str) and sess.history[-1].role == "assistant"
    sess.add_user("again")
    pieces = list(sess.stream_response(cfg=GenerationConfig(max_new_tokens=3, temperature=0.5, seed=1),
                                       effort_tier=2))
    assert len(pieces) <= 3 and len(sess.history) == 5
    assert sess.history[2] == ChatTurn(role="assistant", content=text.strip())


def test_multimodal_prompt_layout():
    from saint_llm_b200.infer import MultimodalSlots

    ids = build_multimodal_prompt_ids([1, 2], [3], MultimodalSlots(9, 7, 8), n_image_pads=2, n_audio_tokens=2)
    assert ids.tolist() == [[1, 2, 9, 9, 7, 7, 7, 8, 3]]


@pytest.mark.parametrize("use_cache", [False, True])
def test_speculative_decode_equals_greedy(model, use_cache):
    ids = _prompt(b=1, t=11)
    torch.manual_seed(3)
    head = EAGLE3DraftHead(model.cfg.hidden_dim, model.cfg.vocab_size, token_conditioned=True)
    out, stats = speculative_decode(model, head, ids, cfg=EAGLE3Config(draft_length=3, max_new_tokens=9,
                                                                        use_cache=use_cache))
    assert torch.equal(out, greedy_decode(model, ids, max_new_tokens=9))
    assert stats["new_tokens"] == 9 and 0.0 <= stats["acceptance_rate"] <= 1.0


def test_speculative_accepts_the_base_models_own_tokens(model):
    ids = _prompt(b=1, t=11)
    greedy = greedy_decode(model, ids, max_new_tokens=30)[0]

    class Oracle(torch.nn.Module):
        """Proposes the base model's greedy continuation (looked up from the previous token's position)."""

        def __init__(self):
            super().__init__()
            self.pos = ids.shape[1]

        def forward(self, hidden, token):
            del hidden
            t = int(token)
            while int(greedy[self.pos]) != t:
                self.pos += 1
            self.pos += 1
            v = torch.full((1, 1, model.cfg.vocab_size), -1e9)
            v[0, 0, int(greedy[min(self.pos, greedy.numel() - 1)])] = 0.0
            return v

    out, stats = speculative_decode(model, Oracle(), ids, cfg=EAGLE3Config(draft_length=4, max_new_tokens=12))
    assert torch.equal(out[0], greedy[:ids.shape[1] + 12])
    assert stats["base_forwards"] < 12


def test_engram_hashing_and_identity():
    cfg = EngramConfig(n_gram=3, n_buckets=97, embedding_dim=8, enabled=True)
    ids = torch.tensor([[5, 6, 7, 8, 9]])
    b = ngram_buckets(ids, 3, 97)
    assert int(b[0, -1]) == trailing_bucket([5, 6, 7, 8, 9], 3, 97) == trailing_bucket([7, 8, 9], 3, 97)
    assert int(b[0, 1]) == trailing_bucket([5, 6], 3, 97)
    table = EngramTable(cfg)
    table.update([7, 8, 9], torch.ones(8))
    assert torch.equal(table.lookup([1, 7, 8, 9]), torch.ones(8))
    hook = EngramHook(16, table)
    h = torch.randn(1, 5, 16)
    assert torch.equal(hook(h, ids), h)  # zero-initialised projection
    torch.nn.init.ones_(hook.proj.weight)
    assert torch.allclose(hook(h, ids)[0, -1], h[0, -1] + 8.0)


def test_multimodal_chat_session_feeds_features_and_records_history():
    from saint_llm_b200.config import MultimodalConfig
    from saint_llm_b200.data.multimodal import TokenSlots
    from saint_llm_b200.data.multimodal_chat import render_multimodal_chat
    from saint_llm_b200.infer.chat import MultimodalChatSession
    from saint_llm_b200.infer.generate import decode
    from saint_llm_b200.infer.sampling import SamplingParams

    m = _model({"multimodal": MultimodalConfig(enable_vision_projector=True, vision_input_dim=8)})
    tok = CharTokenizer(base_vocab=16, unicode_max=480)
    slots = TokenSlots.from_model_config(m.cfg)
    img = torch.randn(3, 8, generator=torch.Generator().manual_seed(4))
    sess = MultimodalChatSession(model=m, tokenizer=tok, slots=slots, system="look")
    with pytest.raises(ValueError):
        sess.add_user()
    sess.add_user("what is it", image_features=[img])
    cfg = GenerationConfig(max_new_tokens=5, temperature=0.0)
    r = render_multimodal_chat(sess.history, tok, slots, add_generation_prompt=True)
    assert r.token_ids.count(slots.image_pad) == 3
    text = sess.respond(cfg=cfg)
    # the same prompt and features decoded without the session (full recomputation)
    want = decode(m, torch.tensor([r.token_ids]), max_new_tokens=5, params=SamplingParams(),
                  eos_token=tok.eos_token_id, vision_features=img)[0, len(r.token_ids):].tolist()
    if tok.eos_token_id in want:
        want = want[:want.index(tok.eos_token_id)]
    assert text == "".join(tok.decode([t]) for t in want)
    assert [t.role for t in sess.history] == ["system", "user", "assistant"]
    assert sess.history[-1].content == tok.decode(want).strip()
    # a different image changes what the model sees
    with torch.no_grad():
        a = m(torch.tensor([r.token_ids]), vision_features=img)["logits"][0, -1]
        b = m(torch.tensor([r.token_ids]), vision_features=img + 1)["logits"][0, -1]
    assert not torch.allclose(a, b)
    sess.reset()
    assert sess.history == []
    with pytest.raises(ValueError):
        next(sess.stream_response(cfg=cfg))
