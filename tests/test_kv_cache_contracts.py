"""Heterogeneous KV cache contracts on CPU: window append / overflow / truncate, compressed
streams emitted exactly at block boundaries (token by token equals all at once), the raw
h-buffer of the unfinished block, rollback rules, and the bundle built for a model."""

import pytest
import torch

from saint_llm_b200.infer.kv_cache import (
    CSAKVCacheLayer,
    HCAKVCacheLayer,
    KVCacheBundle,
    SWAKVCacheLayer,
)


def _mean_blocks(m):
    return lambda raw: raw.view(raw.shape[0], -1, m, raw.shape[-1]).mean(2)


def test_window_append_overflow_truncate():
    c = SWAKVCacheLayer(5, 4, batch_size=2)
    k, v = torch.randn(2, 3, 4), torch.randn(2, 3, 4)
    kk, vv = c.append(k, v)
    assert kk.shape == (2, 3, 4) and torch.equal(kk, k) and torch.equal(vv, v)
    c.append(torch.randn(2, 2, 4), torch.randn(2, 2, 4))
    assert c.length == 5
    with pytest.raises(RuntimeError, match="overflow"):
        c.append(torch.randn(2, 1, 4), torch.randn(2, 1, 4))
    c.truncate(2)
    assert c.length == 2 and torch.equal(c.append(k[:, :1], v[:, :1])[0][:, 2], k[:, 0])
    with pytest.raises(ValueError):
        c.truncate(9)
    assert c.nbytes() == 2 * 2 * 5 * 4 * 4
    c.reset()
    assert c.length == 0
    with pytest.raises(ValueError):
        SWAKVCacheLayer(0, 4)


@pytest.mark.parametrize("keep_history", [False, True])
def test_hca_blocks_emitted_at_boundaries_token_by_token(keep_history):
    m, T, H, D = 4, 11, 6, 3
    h = torch.randn(1, T, H)
    k, v = torch.randn(1, T, D), torch.randn(1, T, D)
    comp = lambda raw: raw.view(1, -1, m, H).mean(2)[..., :D]  # noqa: E731
    one = HCAKVCacheLayer(16, H, D, m, keep_history=keep_history)
    step = HCAKVCacheLayer(16, H, D, m, keep_history=keep_history)
    c1, k1, _ = one.append(h, k, v, compressor=comp)
    for t in range(T):
        c2, k2, _ = step.append(h[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], compressor=comp)
        assert step.n_blocks == (t + 1) // m
        assert step.h_buf_count == (t + 1) % m
    assert torch.equal(c1, c2) and c1.shape[1] == T // m and torch.equal(k1, k2)
    torch.testing.assert_close(c1, h[:, :8].view(1, 2, m, H).mean(2)[..., :D])
    assert torch.equal(step.h_buffer, h[:, 8:11])  # the unfinished block's raw states


def test_compressed_rollback_rules():
    m, H, D = 4, 6, 3
    comp = lambda raw: raw.view(1, -1, m, H).mean(2)[..., :D]  # noqa: E731
    plain = HCAKVCacheLayer(16, H, D, m)
    plain.append(torch.randn(1, 6, H), torch.randn(1, 6, D), torch.randn(1, 6, D), compressor=comp)
    plain.truncate(5)  # inside the unfinished block: fine
    with pytest.raises(RuntimeError, match="keep_history"):
        plain.truncate(3)  # across the emitted block
    hist = HCAKVCacheLayer(16, H, D, m, keep_history=True)
    hist.append(torch.randn(1, 9, H), torch.randn(1, 9, D), torch.randn(1, 9, D), compressor=comp)
    hist.truncate(3)
    assert hist.n_blocks == 0 and hist.length == 3


def test_csa_two_streams_and_compressor_shape_check():
    m, H, D, C = 2, 5, 3, 2
    layer = CSAKVCacheLayer(8, H, D, C, m)
    kv, idx, k, _ = layer.append(torch.randn(1, 5, H), torch.randn(1, 5, D), torch.randn(1, 5, D),
                                 compressor=lambda r: r.view(1, -1, m, H).mean(2)[..., :D],
                                 indexer_compressor=lambda r: r.view(1, -1, m, H).amax(2)[..., :C])
    assert kv.shape == (1, 2, D) and idx.shape == (1, 2, C) and k.shape == (1, 5, D)
    bad = CSAKVCacheLayer(8, H, D, C, m)
    with pytest.raises(RuntimeError, match="compressor returned"):
        bad.append(torch.randn(1, 4, H), torch.randn(1, 4, D), torch.randn(1, 4, D),
                   compressor=lambda r: r[:, :1, :D], indexer_compressor=lambda r: r[:, :2, :C])


def test_bundle_for_model_matches_layer_kinds():
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM

    cfg = ModelConfig.tiny()
    model = SaintLLM(cfg)
    bundle = KVCacheBundle.for_model(model, max_seq_len=64, batch_size=2)
    assert len(bundle) == cfg.n_layers
    kinds = [cfg.layer_kind(i) for i in range(cfg.n_layers)]
    for i, kind in enumerate(kinds):
        layer = bundle.for_layer(i)
        want = {"csa": CSAKVCacheLayer, "hca": HCAKVCacheLayer}.get(kind, SWAKVCacheLayer)
        assert type(layer) is want, (i, kind, type(layer))
    assert bundle.length == 0 and bundle.nbytes() > 0
