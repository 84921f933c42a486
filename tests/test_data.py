"""Data stack on CPU: tokenizers, packing (streaming and native bulk), chat rendering vs
the reference, multimodal packing, corpus mixing, dedup, token shards, BBPE."""

import json

import pytest
import torch

from saint_llm_b200.data import (
    CharTokenizer,
    ChatTurn,
    CorpusSlice,
    MixedCorpus,
    MultimodalChatTurn,
    MultimodalExample,
    ShardedTokenLoader,
    TextFileDataset,
    TokenSlots,
    measure_per_language_fertility,
    pack_flat,
    pack_into_batch,
    pack_multimodal_examples,
    pack_sequences,
    read_token_shard,
    render_chat,
    render_multimodal_chat,
    write_token_shard,
)
from saint_llm_b200.data.pipeline import (
    FingerprintDedup,
    LengthQualityFilter,
    MinHashDedup,
    Pipeline,
    TokenizeStage,
    URLBlocklistFilter,
    minhash_signatures,
)

DOCS = [[5, 6, 7], [], [8], [9, 10, 11, 12, 13], [14, 15]]


def test_char_tokenizer_roundtrip():
    t = CharTokenizer()
    ids = t.encode("héllo ї")
    assert ids[0] == 16 + ord("h") and t.decode([0, 1, *ids, 2]) == "héllo ї"


@pytest.mark.parametrize("drop_last", [True, False])
def test_packing_matches_reference(ref_pkgs, drop_last):
    from saint_llm_data import packing as rp

    for a, b in zip(pack_sequences(DOCS, seq_len=4, eos_token_id=1, drop_last=drop_last),
                    rp.pack_sequences(DOCS, seq_len=4, eos_token_id=1, drop_last=drop_last), strict=True):
        assert torch.equal(a.tokens, b.tokens) and torch.equal(a.segment_ids, b.segment_ids)
    ours = list(pack_into_batch(DOCS, batch_size=3, seq_len=3, eos_token_id=1, drop_last=drop_last))
    theirs = list(rp.pack_into_batch(DOCS, batch_size=3, seq_len=3, eos_token_id=1, drop_last=drop_last))
    assert len(ours) == len(theirs)
    for a, b in zip(ours, theirs, strict=True):
        assert torch.equal(a.tokens, b.tokens) and torch.equal(a.segment_ids, b.segment_ids)


@pytest.mark.parametrize("drop_last", [True, False])
def test_native_bulk_packing_equals_streaming(drop_last):
    flat = torch.tensor([t for d in DOCS for t in d])
    offs = torch.tensor([0, *torch.tensor([len(d) for d in DOCS]).cumsum(0).tolist()])
    bulk = pack_flat(flat, offs, seq_len=4, eos_token_id=1, pad_token_id=0, drop_last=drop_last)
    stream = list(pack_sequences(DOCS, seq_len=4, eos_token_id=1, drop_last=drop_last))
    assert torch.equal(bulk.tokens, torch.cat([w.tokens for w in stream]))
    assert torch.equal(bulk.segment_ids, torch.cat([w.segment_ids for w in stream]))


def _turns():
    return [ChatTurn("system", "sys"), ChatTurn("user", "hi"),
            ChatTurn("assistant", "ok", thinking="hmm", effort_tier=2), ChatTurn("user", "more")]


@pytest.mark.parametrize("kw", [{}, {"add_generation_prompt": True}, {"append_eos": True, "mask_thinking": False}])
def test_chat_render_matches_reference(ref_pkgs, kw):
    from saint_llm_data import chat_template as rc
    from saint_llm_data.tokenizer import CharTokenizer as RT

    ours = render_chat(_turns(), CharTokenizer(), **kw)
    theirs = rc.render_chat([rc.ChatTurn(t.role, t.content, t.thinking, t.effort_tier) for t in _turns()], RT(),
                            **kw)
    assert ours.token_ids == theirs.token_ids and ours.loss_mask == theirs.loss_mask and ours.text == theirs.text


def test_multimodal_chat_matches_reference(ref_pkgs):
    from saint_llm_data import multimodal as rmm
    from saint_llm_data import multimodal_chat as rmc
    from saint_llm_data.tokenizer import CharTokenizer as RT

    img, aud = torch.randn(3, 4), torch.randn(2, 5)
    turns = [MultimodalChatTurn("user", "see", image_features=(img,), audio_features=(aud,)),
             MultimodalChatTurn("assistant", "yes")]
    ours = render_multimodal_chat(turns, CharTokenizer(), TokenSlots(3, 4, 5), append_eos=True)
    theirs = rmc.render_multimodal_chat(
        [rmc.MultimodalChatTurn(t.role, t.content, image_features=t.image_features, audio_features=t.audio_features)
         for t in turns], RT(), rmm.TokenSlots(3, 4, 5), append_eos=True)
    assert ours.token_ids == theirs.token_ids and ours.loss_mask == theirs.loss_mask
    assert torch.equal(ours.vision_features, theirs.vision_features)
    assert torch.equal(ours.audio_features, theirs.audio_features)


def test_multimodal_packing_keeps_features_aligned_with_slots():
    slots = TokenSlots(image_pad=3, audio_start=4, audio_end=5)
    tok = CharTokenizer()
    exs = [MultimodalExample("a", "b", image_features=(torch.ones(3, 2),)),
           MultimodalExample("c", "d", image_features=(2 * torch.ones(2, 2),), audio_features=(torch.ones(1, 6),))]
    wins = list(pack_multimodal_examples(exs, tok, slots, seq_len=4, drop_last=False))
    n_img = sum(int((w.tokens == 3).sum()) for w in wins)
    assert n_img == 5 and sum(0 if w.vision_features is None else w.vision_features.shape[0] for w in wins) == 5
    for w in wins:
        k = int((w.tokens == 3).sum())
        assert (w.vision_features is None and k == 0) or w.vision_features.shape[0] == k
        a = int(((w.tokens >= 4) & (w.tokens <= 5)).sum())
        assert (w.audio_features is None and a == 0) or w.audio_features.shape[0] == a


def test_mixed_corpus_and_fertility():
    mc = MixedCorpus([CorpusSlice("a", 3.0, ["a"] * 50), CorpusSlice("b", 1.0, ["b"] * 5)], seed=0)
    out = list(mc)
    assert len(out) == 55 and out.count("b") == 5 and mc.counts == {"a": 50, "b": 5}
    assert len(list(MixedCorpus([CorpusSlice("a", 1.0, ["x"] * 9)], max_docs=4))) == 4
    rep = measure_per_language_fertility(CharTokenizer(), {"uk": ["привіт"], "en": ["", "hi"]})
    assert [r.language for r in rep.records] == ["en", "uk"] and rep.by_language()["uk"].fertility == 1.0
    with pytest.raises(ValueError):
        MixedCorpus([CorpusSlice("a", 0.0, [])])


def test_pipeline_dedup_and_filters():
    docs = [{"text": "the quick brown fox jumps", "language": "en"},
            {"text": "the quick brown fox jumps", "language": "en"},
            {"text": "the quick brown fox jumped", "language": "en"},
            {"text": "tiny", "language": "en"},
            {"text": "ukrainian text that is long enough", "language": "uk",
             "meta": {"url": "https://auto-translate.example/a"}}]
    p = Pipeline([LengthQualityFilter(min_chars=10), FingerprintDedup(), MinHashDedup(n_perm=32),
                  URLBlocklistFilter(), TokenizeStage(CharTokenizer())])
    kept, drops = p.stats_run(docs)
    assert len(kept) == 2 and drops == {"length_quality_filter": 1, "fingerprint_dedup": 1, "minhash_dedup": 0,
                                        "url_blocklist": 1, "tokenize": 0}
    assert kept[0]["token_ids"][0] == 16 + ord("t")
    s = minhash_signatures(["abcdefgh", "abcdefgh", "zzzzzzzz", ""], n_perm=16)
    assert torch.equal(s[0], s[1]) and not torch.equal(s[0], s[2]) and int(s[3].abs().sum()) == 0
    same = minhash_signatures(["abcdefghij" * 20, "abcdefghij" * 20 + "x"], n_perm=256)
    assert (same[0] == same[1]).float().mean() > 0.8  # Jaccard ~ 0.99


def test_token_shards_and_native_loader(tmp_path):
    toks = torch.arange(1000) % 700
    p1 = write_token_shard(tmp_path / "a.bin", toks[:600], vocab_size=700)
    p2 = write_token_shard(tmp_path / "b.bin", toks[600:], vocab_size=70000)
    assert torch.equal(torch.from_numpy(read_token_shard(p1).astype("int64")), toks[:600])
    ld = ShardedTokenLoader([p1, p2], batch_size=3, seq_len=16, seed=7, prefetch=2)
    assert ld.total_windows == (600 - 16) + (400 - 16)
    first = [ld.next() for _ in range(4)]
    ld.close()
    for b in first:
        assert b.shape == (3, 16)
        for row in b:  # every row is a contiguous run of the corpus
            assert bool(((row[1:] - row[:-1]) % 700 == 1).all())
    again = ShardedTokenLoader([p1, p2], batch_size=3, seq_len=16, seed=7, prefetch=3)
    second = [again.next() for _ in range(4)]
    again.close()
    assert all(torch.equal(a, b) for a, b in zip(first, second, strict=True))
    other = ShardedTokenLoader([p1, p2], batch_size=3, seq_len=16, seed=7, rank=1, world_size=2)
    assert not torch.equal(other.next(), first[0])
    other.close()


def test_text_file_dataset(tmp_path):
    f = tmp_path / "d.jsonl"
    f.write_text("\n".join(json.dumps({"text": t}) for t in ["ab", "cde", "f"]) + "\n")
    batches = list(TextFileDataset(f, CharTokenizer(), seq_len=4, batch_size=2, jsonl=True, drop_last=False))
    assert batches[0].tokens.shape == (2, 4) and int(batches[0].tokens[0, 2]) == 1


def test_train_bbpe(tmp_path):
    from saint_llm_b200.data import SAINT_V0_0_SPECIAL_TOKENS, train_bbpe

    corpus = ["привіт світ hello world"] * 50 + ["the cat sat on the mat"] * 50
    tok = train_bbpe(corpus, tmp_path / "tok.json", vocab_size=300, special_tokens=SAINT_V0_0_SPECIAL_TOKENS)
    assert tok.eos_token_id == 1 and tok.pad_token_id == 0
    assert tok.decode(tok.encode("hello world")) == "hello world"
    assert tok.token_to_id("<|effort:3|>") == SAINT_V0_0_SPECIAL_TOKENS.index("<|effort:3|>")
