"""The engine's candidate-sampling path on the B200 (eager decode with the
per-slot logit rewrite): invariants that hold whatever the bf16 rounding --
allowed_token_ids bounds the output, a large logit_bias forces its token,
bad_words bans it, min_tokens masks a stop token until enough tokens exist,
a stop token retires the request, a grammar's output is in its language."""
import pytest
import torch

from vllm_sm70_b200.engine import LLM, SamplingParams, StructuredOutputsParams

from .test_engine_gpu import SMALL

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def llm():
    from .test_structured_cpu import _tokenizer

    eng = LLM(SMALL, max_num_seqs=8, max_model_len=256, seed=11, tokenizer=_tokenizer())
    yield eng
    eng.shutdown()


def _prompts(n=4):
    g = torch.Generator().manual_seed(21)
    return [torch.randint(0, 256, (L,), generator=g) for L in (9, 33, 17, 60)[:n]]


def test_allowed_bias_bad_words(b200_ops, llm):
    a = llm.get_tokenizer().encode("a", add_special_tokens=False)[0]
    allowed = [65, 66, 67, 300, 4000]
    outs = llm.generate(_prompts(), SamplingParams(max_tokens=8, ignore_eos=True, temperature=1.0,
                                                   seed=4, allowed_token_ids=allowed))
    assert all(set(o.output_token_ids) <= set(allowed) for o in outs)
    forced = llm.generate(_prompts(), SamplingParams(max_tokens=6, ignore_eos=True,
                                                     logit_bias={a: 1e4}))
    assert all(o.output_token_ids == [a] * 6 for o in forced)
    banned = llm.generate(_prompts(), SamplingParams(max_tokens=6, ignore_eos=True,
                                                     logit_bias={a: 1e4}, bad_words=["a"]))
    assert all(a not in o.output_token_ids and len(o.output_token_ids) == 6 for o in banned)


def test_stop_and_min_tokens(b200_ops, llm):
    sp = SamplingParams(max_tokens=20, stop_token_ids=[98], logit_bias={98: 1e4})
    assert all(o.output_token_ids == [98] and o.finish_reason == "stop"
               for o in llm.generate(_prompts(), sp))
    sp = SamplingParams(max_tokens=20, stop_token_ids=[98], logit_bias={98: 1e4}, min_tokens=3)
    for o in llm.generate(_prompts(), sp):
        assert len(o.output_token_ids) == 4 and o.output_token_ids[-1] == 98
        assert 98 not in o.output_token_ids[:3]


def test_grammar_output(b200_ops, llm):
    so = StructuredOutputsParams(choice=["north", "south", "east"])
    sp = SamplingParams(max_tokens=24, temperature=0.8, seed=2, structured_outputs=so)
    for o in llm.generate(_prompts(), sp):
        assert o.outputs[0].text in ("north", "south", "east"), o.outputs[0].text
        assert o.outputs[0].finish_reason == "stop"
