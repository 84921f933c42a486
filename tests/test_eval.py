"""Perplexity and the harness adapter vs the unmodified reference on the same weights (CPU)."""

from dataclasses import dataclass

import pytest
import torch

from saint_llm_b200.config import ModelConfig
from saint_llm_b200.data import CharTokenizer
from saint_llm_b200.eval import SaintLLMHarnessLM, compute_perplexity, compute_perplexity_streaming
from saint_llm_b200.models import SaintLLM


@dataclass
class Req:
    args: tuple


@pytest.fixture(scope="module")
def pair(ref_pkgs):
    from saint_llm_core.config import ModelConfig as RC
    from saint_llm_core.model import SaintLLM as RM

    torch.manual_seed(0)
    ours = SaintLLM(ModelConfig.tiny()).eval()
    torch.manual_seed(0)
    ref = RM(RC.tiny()).eval()
    ref.load_state_dict(ours.state_dict())
    return ours, ref


def test_perplexity_matches_reference(pair):
    from saint_llm_eval.perplexity import compute_perplexity as rp
    from saint_llm_eval.perplexity import compute_perplexity_streaming as rps

    ours, ref = pair
    ids = torch.randint(0, 512, (2, 20), generator=torch.Generator().manual_seed(1))
    ids2 = ids.clone()
    ids2[0, 5] = -100
    assert compute_perplexity(ours, ids) == pytest.approx(rp(ref, ids), rel=1e-5)
    # labels equal to ignore_index are skipped (the reference would also feed -100 to the embedding)
    p_ign = compute_perplexity(ours, ids2)
    assert p_ign != compute_perplexity(ours, ids) and p_ign < float("inf")
    batches = [ids, ids[:, :7]]
    assert compute_perplexity_streaming(ours, batches) == pytest.approx(rps(ref, batches), rel=1e-5)


def test_harness_matches_reference(pair):
    from saint_llm_data.tokenizer import CharTokenizer as RT
    from saint_llm_eval.harness.saint_llm_lm import SaintLLMHarnessLM as RH

    ours, ref = pair
    tok, rtok = CharTokenizer(base_vocab=16, unicode_max=496), RT(base_vocab=16, unicode_max=496)
    a = SaintLLMHarnessLM(model=ours, tokenizer=tok, batch_size=2)
    b = RH(model=ref, tokenizer=rtok)
    reqs = [Req(("hello wor", "ld")), Req(("ab", "")), Req(("x", "yz!"))]
    for (la, ga), (lb, gb) in zip(a.loglikelihood(reqs), b.loglikelihood(reqs), strict=True):
        assert la == pytest.approx(lb, rel=1e-4, abs=1e-4) and ga == gb
    rolls = [Req(("some text",)), Req(("q",))]
    assert a.loglikelihood_rolling(rolls) == pytest.approx(b.loglikelihood_rolling(rolls), rel=1e-4, abs=1e-4)
    gen = [Req(("abc", {"until": ["\n"], "max_gen_toks": 4}))]
    assert a.generate_until(gen) == b.generate_until(gen)


class _Req:
    def __init__(self, *args):
        self.args = args


def _tiny():
    from saint_llm_b200.config import ModelConfig
    from saint_llm_b200.models import SaintLLM

    torch.manual_seed(0)
    return SaintLLM(ModelConfig.tiny()).eval()


def test_perplexity_masking_streaming_and_errors():
    import math

    from saint_llm_b200.eval.perplexity import compute_perplexity, compute_perplexity_streaming, token_nll

    m = _tiny()
    ids = torch.randint(0, 500, (2, 12))
    ppl = compute_perplexity(m, ids)
    assert 1.0 < ppl < 5000.0
    s, n = token_nll(m, ids)
    assert int(n) == 22 and math.isclose(ppl, math.exp(float(s) / 22), rel_tol=1e-5)
    masked = ids.clone()
    masked[:, 6:] = -100
    s2, n2 = token_nll(m, masked)
    assert int(n2) == 10
    # streaming over two halves of the batch equals the batch
    assert math.isclose(compute_perplexity_streaming(m, [ids[:1], ids[1:], ids[:, :1]]), ppl, rel_tol=1e-5)
    nothing_scored = torch.tensor([[3, -100, -100, -100]])
    assert compute_perplexity(m, nothing_scored) == math.inf
    assert compute_perplexity_streaming(m, []) == math.inf
    with pytest.raises(ValueError):
        compute_perplexity(m, ids[0])
    with pytest.raises(ValueError):
        compute_perplexity(m, ids[:, :1])


def test_harness_loglikelihood_contract():
    from saint_llm_b200.data.tokenizer import CharTokenizer
    from saint_llm_b200.eval.harness import SaintLLMHarnessLM

    lm = SaintLLMHarnessLM(model=_tiny(), tokenizer=CharTokenizer())
    res = lm.loglikelihood([_Req("abc", "de"), _Req("abc", ""), _Req("x", "y")])
    assert len(res) == 3 and res[1] == (0.0, True)
    assert res[0][0] < 0 and isinstance(res[0][1], bool)
    rolling = lm.loglikelihood_rolling([_Req("hello"), _Req("h")])
    assert rolling[1] == 0.0 and rolling[0] < 0
    # the continuation's log-likelihood equals the rolling score difference of the two texts
    full = lm.loglikelihood_rolling([_Req("abcde")])[0]
    ctx = lm.loglikelihood_rolling([_Req("abc")])[0]
    assert abs((full - ctx) - res[0][0]) < 1e-3
