"""Static-shape decoding (ring window cache, device-side positions, pooled compressed
entries) against the cached decode path: same logits every step (CPU, fp32)."""

import pytest
import torch


@pytest.mark.parametrize("upd,prompt,chunk", [({}, 13, 5), ({}, 16, 16),
                                              ({"final_logit_softcap": 20.0}, 9, 4)])
def test_static_decoder_matches_cached_path(upd, prompt, chunk):
    """The indexer keeps every visible block (top-k larger than the block count): with
    ReLU'd scores many blocks tie at 0 and ``topk`` may break ties differently on score
    vectors of different lengths, which is not a difference of the two paths."""
    from saint_llm_b200.config import CSAConfig, ModelConfig
    from saint_llm_b200.infer.generate import last_logits
    from saint_llm_b200.infer.kv_cache import KVCacheBundle
    from saint_llm_b200.infer.static_decode import StaticDecoder
    from saint_llm_b200.models import SaintLLM

    base = ModelConfig.tiny()
    csa = CSAConfig(**{**base.csa.model_dump(), "attention_top_k": 64})
    cfg = base.model_copy(update={**upd, "csa": csa})
    torch.manual_seed(0)
    model = SaintLLM(cfg).eval()
    with torch.no_grad():  # sharper logits than the default init, so argmax is not degenerate
        for blk in model.blocks:
            blk.attention.sink_logit.normal_()
    x = torch.randint(0, cfg.vocab_size, (2, prompt))
    steps = 14
    with torch.no_grad():
        ref = KVCacheBundle.for_model(model, max_seq_len=prompt + steps, batch_size=2)
        st_bundle = KVCacheBundle.for_model(model, max_seq_len=prompt + steps, batch_size=2)
        lg = last_logits(model, x, bundle=ref)
        lg2 = None
        for c in range(0, prompt, chunk):
            lg2 = last_logits(model, x[:, c:c + chunk], bundle=st_bundle)
        torch.testing.assert_close(lg2, lg, atol=1e-4, rtol=1e-4)
        dec = StaticDecoder(model, 2, prompt + steps)
        dec.load(st_bundle, lg2)
        tok = lg.argmax(-1, keepdim=True)
        for i in range(steps):
            assert torch.equal(dec.tok, tok), i
            dec._step()
            want = last_logits(model, tok, bundle=ref)
            torch.testing.assert_close(dec.logits, want.float(), atol=1e-4, rtol=1e-4, msg=f"step {i}")
            tok = want.argmax(-1, keepdim=True)
            dec.tok.copy_(dec.next_tok)


def test_static_greedy_decode_api():
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.infer import greedy_decode_cached
    from saint_llm_b200.infer.static_decode import static_greedy_decode
    from saint_llm_b200.models import SaintLLM

    cfg = ModelConfig.tiny()
    torch.manual_seed(1)
    model = SaintLLM(cfg).eval()
    x = torch.randint(0, cfg.vocab_size, (3, 11))
    assert torch.equal(static_greedy_decode(model, x, max_new_tokens=10, prefill_chunk=4),
                       greedy_decode_cached(model, x, max_new_tokens=10))


@pytest.mark.gpu
def test_cuda_graph_decode_matches_eager_static(cuda):
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.infer.generate import last_logits
    from saint_llm_b200.infer.kv_cache import KVCacheBundle
    from saint_llm_b200.infer.static_decode import StaticDecoder
    from saint_llm_b200.models import SaintLLM
    from saint_llm_b200.train.engine import cast_params

    cfg = ModelConfig.bench_16b().model_copy(update={"n_layers": 3, "linear_quant": "bf16"})
    torch.manual_seed(0)
    with torch.device(cuda):
        model = SaintLLM(cfg)
    cast_params(model)
    model.eval()
    x = torch.randint(0, cfg.vocab_size, (4, 300), device=cuda)
    outs = []
    for graph in (False, True):
        with torch.no_grad():
            bundle = KVCacheBundle.for_model(model, max_seq_len=340, batch_size=4)
            lg = None
            for c in range(0, 300, 128):
                lg = last_logits(model, x[:, c:c + 128], bundle=bundle)
            dec = StaticDecoder(model, 4, 340)
            dec.load(bundle, lg)
            if graph:
                dec.capture()
            outs.append(dec.generate(24))
    assert torch.equal(outs[0], outs[1])
