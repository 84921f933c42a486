"""Data-path contracts on CPU: packing invariants (streaming vs native bulk), batch padding,
corpus mixing, the document pipeline, MinHash behaviour and the native shard loader."""

import random

import pytest
import torch

from saint_llm_b200.data import pack_into_batch, pack_sequences
from saint_llm_b200.data.mix_corpus import CorpusSlice, MixedCorpus
from saint_llm_b200.data.packing import pack_flat
from saint_llm_b200.data.pipeline.dedup import FingerprintDedup, MinHashDedup, minhash_signatures
from saint_llm_b200.data.pipeline.filters import LengthQualityFilter, QualityFilter
from saint_llm_b200.data.pipeline.stage import Pipeline
from saint_llm_b200.data.token_loader import ShardedTokenLoader, read_token_shard, write_token_shard


def _docs(n, seed=0, lo=1, hi=40):
    rng = random.Random(seed)
    return [[rng.randrange(5, 100) for _ in range(rng.randrange(lo, hi))] for _ in range(n)]


@pytest.mark.parametrize("seq_len", [1, 7, 64])
def test_packing_preserves_the_stream(seq_len):
    """Concatenating the windows (drop_last=False, padding stripped) gives back every document
    followed by EOS, and segment ids count documents in order."""
    docs = _docs(30, seed=seq_len)
    eos, pad = 1, 0
    wins = list(pack_sequences(docs, seq_len=seq_len, eos_token_id=eos, pad_token_id=pad, drop_last=False))
    assert all(w.shape == (1, seq_len) for w in wins)
    stream = torch.cat([w.tokens[0] for w in wins])
    segs = torch.cat([w.segment_ids[0] for w in wins])
    want = torch.tensor([t for d in docs for t in d + [eos]])
    n = want.numel()
    assert torch.equal(stream[:n], want)
    assert (stream[n:] == pad).all()
    want_seg = torch.tensor([i for i, d in enumerate(docs) for _ in range(len(d) + 1)])
    assert torch.equal(segs[:n], want_seg)
    assert (segs[n:] == want_seg[-1]).all()  # padding keeps the last document's id


def test_packing_drop_last_and_empty_docs():
    docs = [[5, 6, 7], [], [8]]  # the empty document is skipped entirely
    wins = list(pack_sequences(docs, seq_len=4, eos_token_id=1))
    assert len(wins) == 1 and wins[0].tokens.tolist() == [[5, 6, 7, 1]]
    assert wins[0].segment_ids.tolist() == [[0, 0, 0, 0]]
    with pytest.raises(ValueError, match="seq_len must be positive"):
        list(pack_sequences(docs, seq_len=0, eos_token_id=1))


def test_batches_pad_rows_with_segment_minus_one():
    docs = _docs(9, seed=3, lo=5, hi=9)
    batches = list(pack_into_batch(docs, batch_size=4, seq_len=8, eos_token_id=1, pad_token_id=0, drop_last=False))
    assert all(b.shape == (4, 8) for b in batches)
    last = batches[-1]
    pad_rows = (last.segment_ids == -1).all(dim=1)
    assert pad_rows.any() and (last.tokens[pad_rows] == 0).all()
    full = list(pack_into_batch(docs, batch_size=4, seq_len=8, eos_token_id=1, drop_last=True))
    assert all(not (b.segment_ids == -1).any() for b in full)


@pytest.mark.parametrize("drop_last", [True, False])
def test_native_bulk_packing_matches_streaming_on_random_corpus(drop_last):
    docs = _docs(200, seed=11, lo=1, hi=300)
    flat = torch.tensor([t for d in docs for t in d])
    offs = torch.tensor([0] + list(torch.tensor([len(d) for d in docs]).cumsum(0)))
    bulk = pack_flat(flat, offs, seq_len=128, eos_token_id=2, pad_token_id=0, drop_last=drop_last)
    stream = list(pack_sequences(docs, seq_len=128, eos_token_id=2, pad_token_id=0, drop_last=drop_last))
    assert torch.equal(bulk.tokens, torch.cat([w.tokens for w in stream]))
    assert torch.equal(bulk.segment_ids, torch.cat([w.segment_ids for w in stream]))


def test_mixed_corpus_weights_exhaustion_and_limits():
    mix = MixedCorpus([CorpusSlice("a", 3.0, [f"a{i}" for i in range(3000)]),
                       CorpusSlice("b", 1.0, [f"b{i}" for i in range(3000)])], max_docs=2000, seed=0)
    out = list(mix)
    assert len(out) == 2000
    frac_a = mix.counts["a"] / 2000
    assert 0.70 < frac_a < 0.80, frac_a
    # a short slice drops out and the rest continues until everything is used
    mix2 = MixedCorpus([CorpusSlice("s", 100.0, ["s0", "s1"]), CorpusSlice("l", 1.0, [f"l{i}" for i in range(50)])])
    out2 = list(mix2)
    assert sorted(out2) == sorted(["s0", "s1"] + [f"l{i}" for i in range(50)])
    for bad in ([], [CorpusSlice("z", 0.0, [])]):
        with pytest.raises(ValueError):
            MixedCorpus(bad)


def test_pipeline_counts_drops_per_stage():
    class Score:
        def __call__(self, text, *, language=None):
            return 1.0 if "good" in text else 0.0

    docs = [{"text": "good " * 30}, {"text": "bad " * 30}, {"text": "good"}, {"text": "good " * 30}]
    pipe = Pipeline([LengthQualityFilter(min_chars=20), QualityFilter(Score(), 0.5), FingerprintDedup()])
    kept, drops = pipe.stats_run(docs)
    assert [d["text"] for d in kept] == ["good " * 30]
    assert drops == {"length_quality_filter": 1, "quality_filter": 1, "fingerprint_dedup": 1} or \
        sum(drops.values()) == 3


def test_minhash_similarity_tracks_overlap():
    base = "the quick brown fox jumps over the lazy dog " * 8
    near = base.replace("lazy", "sleepy", 1)
    other = "completely different text about tensor cores and memory bandwidth " * 6
    sig = minhash_signatures([base, near, other], n_perm=256)
    agree = lambda i, j: (sig[i] == sig[j]).float().mean().item()  # noqa: E731
    assert agree(0, 1) > 0.7 and agree(0, 2) < 0.2
    assert torch.equal(sig, minhash_signatures([base, near, other], n_perm=256))  # deterministic
    d = MinHashDedup()  # drops documents whose whole signature repeats
    kept = d.filter_batch([{"text": base}, {"text": other}, {"text": base}, {"text": ""}, {"text": near}])
    assert [k["text"] for k in kept] == [base, other, "", near]
    assert d({"text": other}) is None and len(d) == 3


def test_shard_loader_windows_are_deterministic_and_rank_disjoint(tmp_path):
    toks = torch.arange(20_000) % 997
    paths = [write_token_shard(tmp_path / f"s{i}.bin", toks[i * 10_000:(i + 1) * 10_000], vocab_size=997)
             for i in range(2)]
    assert torch.equal(torch.from_numpy(read_token_shard(paths[1]).astype("int64")), toks[10_000:])

    def draw(rank, world, seed, n=6):
        ld = ShardedTokenLoader(paths, batch_size=2, seq_len=64, seed=seed, rank=rank, world_size=world)
        try:
            return [ld.next().clone() for _ in range(n)]
        finally:
            ld.close()

    a, b = draw(0, 1, 7), draw(0, 1, 7)
    assert all(torch.equal(x, y) for x, y in zip(a, b, strict=True))
    for x in a:  # every row is a contiguous window of one shard
        assert x.shape == (2, 64) and ((x[:, 1:] - x[:, :-1]) % 997 == 1).all()
    r0, r1 = draw(0, 2, 7), draw(1, 2, 7)
    starts0 = {int(r[0]) for x in r0 for r in x}
    starts1 = {int(r[0]) for x in r1 for r in x}
    assert r0[0].shape == (2, 64) and starts0 != starts1
