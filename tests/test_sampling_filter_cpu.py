"""Top-k / top-p sampling on CPU: the candidate sampler's oracle follows the
kernel's rules (ordering, top-k cut, nucleus prefix, greedy at T <= 0, a
distribution proportional to softmax over the kept set), and the engine
routes requests with top-k / top-p through it: top_k = 1 and a vanishing
top_p reduce to greedy decoding, a fixed seed is reproducible, and greedy
requests batched with filtered ones are unchanged."""
import pytest
import torch

from vllm_sm70_b200.engine import SamplingParams
from vllm_sm70_b200.ops import sampling

from .test_engine_cpu import _llm


def _cands(rows, C):
    v = torch.linspace(3, -3, C).expand(rows, C).contiguous()
    i = torch.arange(C, dtype=torch.int32).expand(rows, C).contiguous()
    perm = torch.randperm(C, generator=torch.Generator().manual_seed(0))
    return v[:, perm].contiguous(), i[:, perm].contiguous()   # unsorted input


def test_oracle_rules():
    rows, C = 200, 16
    v, i = _cands(rows, C)
    t = torch.ones(rows)
    seeds = torch.arange(rows, dtype=torch.int64)
    k = torch.full((rows,), 3, dtype=torch.int32)
    p = torch.ones(rows)
    out = sampling.sample_candidates(v, i, t, k, p, seeds, 0)
    assert int(out.max()) < 3 and int(out.min()) >= 0 and len(set(out.tolist())) == 3
    k.fill_(-1)
    p.fill_(0.5)
    out = sampling.sample_candidates(v, i, t, k, p, seeds, 1)
    probs = torch.softmax(torch.linspace(3, -3, C), 0)
    keep = int((torch.cumsum(probs, 0) < 0.5).sum()) + 1
    assert int(out.max()) < keep
    t.fill_(0.0)
    assert sampling.sample_candidates(v, i, t, k, p, seeds, 2).tolist() == [0] * rows
    # absent candidates (id < 0) are never picked; none at all -> -1
    i2 = i.clone()
    i2[:, :] = -1
    assert sampling.sample_candidates(v, i2, torch.ones(rows), k, torch.ones(rows), seeds,
                                      3).tolist() == [-1] * rows


def test_oracle_distribution():
    rows, C = 6000, 4
    v = torch.tensor([1.0, 0.5, 0.0, -4.0]).expand(rows, C).contiguous()
    i = torch.arange(C, dtype=torch.int32).expand(rows, C).contiguous()
    out = sampling.sample_candidates(v, i, torch.ones(rows), torch.full((rows,), 3, dtype=torch.int32),
                                     torch.ones(rows), torch.arange(rows, dtype=torch.int64), 7)
    freq = torch.bincount(out.to(torch.int64), minlength=C).float() / rows
    want = torch.softmax(torch.tensor([1.0, 0.5, 0.0]), 0)
    assert freq[3] == 0
    assert torch.allclose(freq[:3], want, atol=0.03), (freq, want)


def _prompts():
    g = torch.Generator().manual_seed(4)
    return [torch.randint(0, 512, (n,), generator=g) for n in (7, 21, 12)]


def test_engine_filtered_requests():
    llm = _llm()
    greedy = [o.output_token_ids for o in llm.generate(_prompts(), SamplingParams(max_tokens=5))]
    k1 = llm.generate(_prompts(), SamplingParams(max_tokens=5, temperature=1.0, top_k=1))
    assert [o.output_token_ids for o in k1] == greedy
    p0 = llm.generate(_prompts(), SamplingParams(max_tokens=5, temperature=1.0, top_p=1e-9, seed=2))
    assert [o.output_token_ids for o in p0] == greedy
    sp = SamplingParams(max_tokens=5, temperature=1.5, top_k=20, top_p=0.9, seed=11)
    a = [o.output_token_ids for o in llm.generate(_prompts(), sp)]
    b = [o.output_token_ids for o in llm.generate(_prompts(), sp)]
    assert a == b and all(len(t) == 5 for t in a)
    mixed = llm.generate(_prompts(), [SamplingParams(max_tokens=5), sp, SamplingParams(max_tokens=5)])
    assert mixed[0].output_token_ids == greedy[0] and mixed[2].output_token_ids == greedy[2]
    assert not llm.runner.filtering  # reset after the call


def _penalized_greedy(model, prompt, n, rep=1.0, pres=0.0, freq=0.0):
    """Greedy decoding with vLLM's penalty rules on a dense forward."""
    from ._llama_ref import llama_logits

    ids, out = prompt.clone(), []
    for _ in range(n):
        lg = llama_logits(model, ids)[-1].clone()
        counts = torch.bincount(torch.tensor(out, dtype=torch.int64), minlength=lg.numel()).float() \
            if out else torch.zeros_like(lg)
        seen = counts > 0
        pseen = torch.zeros_like(lg, dtype=torch.bool)
        pseen[prompt] = True
        m = seen | pseen
        lg = torch.where(m, torch.where(lg > 0, lg / rep, lg * rep), lg)
        lg = lg - freq * counts - pres * seen.float()
        t = int(lg.argmax())
        out.append(t)
        ids = torch.cat([ids, torch.tensor([t])])
    return out


def test_penalties_match_dense_reference():
    """repetition / presence / frequency penalties (greedy) equal a dense
    reference applying vLLM's rules; a request without penalties in the same
    batch is unchanged; penalties change the output of a repetitive prompt."""
    llm = _llm()
    p = torch.tensor([5, 9, 5, 9, 5, 9, 5, 9, 7, 7, 7, 7])
    plain = llm.generate([p], SamplingParams(max_tokens=8))[0].output_token_ids
    for kw in (dict(repetition_penalty=1.8), dict(presence_penalty=2.0),
               dict(frequency_penalty=1.5), dict(repetition_penalty=1.3, frequency_penalty=0.7)):
        sp = SamplingParams(max_tokens=8, **kw)
        got = llm.generate([p, p], [sp, SamplingParams(max_tokens=8)])
        want = _penalized_greedy(llm.model, p, 8, kw.get("repetition_penalty", 1.0),
                                 kw.get("presence_penalty", 0.0), kw.get("frequency_penalty", 0.0))
        assert got[0].output_token_ids == want, kw
        assert got[1].output_token_ids == plain
    strong = llm.generate([p], SamplingParams(max_tokens=8, frequency_penalty=50.0))[0]
    assert len(set(strong.output_token_ids)) == 8  # every repeat is penalised away


def test_min_p_keeps_only_likely_tokens():
    """Every token sampled with ``min_p`` is in its step's min_p set
    (probability >= min_p x the top one, i.e. logit >= max + T log min_p),
    checked against a dense teacher-forced forward; min_p = 1 is greedy."""
    import math

    from ._llama_ref import llama_logits

    llm = _llm()
    T, mp = 1.0, 0.5

    def violations(sp):
        n = 0
        for p, o in zip(_prompts(), llm.generate(_prompts(), sp)):
            seq = torch.cat([p, torch.tensor(o.output_token_ids)])
            for k, tok in enumerate(o.output_token_ids):
                lg = llama_logits(llm.model, seq[: p.numel() + k])[-1]
                n += float(lg[tok]) < float(lg.max()) + T * math.log(mp) - 1e-4
        return n

    assert violations(SamplingParams(max_tokens=6, temperature=T, min_p=mp, seed=5)) == 0
    assert violations(SamplingParams(max_tokens=6, temperature=T, seed=5)) > 0  # discriminates
    greedy = [o.output_token_ids for o in llm.generate(_prompts(), SamplingParams(max_tokens=5))]
    top = SamplingParams(max_tokens=5, temperature=2.0, min_p=1.0, seed=3)
    assert [o.output_token_ids for o in llm.generate(_prompts(), top)] == greedy


def test_logit_bias_and_allowed_token_ids():
    """``allowed_token_ids`` limits greedy decoding to the set and
    ``logit_bias`` is added to the logits (vLLM's order: mask, then bias, then
    penalties); both equal a dense reference that applies them, requests
    without them in the same batch are unchanged, a large bias forces its
    token, and ids outside the vocabulary are refused."""
    from ._llama_ref import llama_logits

    llm = _llm()
    p = _prompts()[1]
    plain = llm.generate([p], SamplingParams(max_tokens=6))[0].output_token_ids

    def dense(n, allowed=None, bias=None, rep=1.0):
        ids, out = p.clone(), []
        for _ in range(n):
            lg = llama_logits(llm.model, ids)[-1].clone()
            if allowed is not None:
                keep = torch.zeros_like(lg, dtype=torch.bool)
                keep[allowed] = True
                lg = torch.where(keep, lg, torch.full_like(lg, float("-inf")))
            for t, v in (bias or {}).items():
                lg[t] += v
            seen = torch.zeros_like(lg, dtype=torch.bool)
            seen[ids] = True
            lg = torch.where(seen, torch.where(lg > 0, lg / rep, lg * rep), lg)
            t = int(lg.argmax())
            out.append(t)
            ids = torch.cat([ids, torch.tensor([t])])
        return out

    allowed = [3, 17, 42, 99, 250, 511]
    got = llm.generate([p, p], [SamplingParams(max_tokens=6, allowed_token_ids=allowed),
                                SamplingParams(max_tokens=6)])
    assert got[0].output_token_ids == dense(6, allowed=allowed)
    assert set(got[0].output_token_ids) <= set(allowed)
    assert got[1].output_token_ids == plain
    bias = {plain[0]: -1e4, 77: 3.0}
    sp = SamplingParams(max_tokens=6, logit_bias=bias, repetition_penalty=1.5)
    got = llm.generate([p], sp)[0].output_token_ids
    assert got == dense(6, bias=bias, rep=1.5) and plain[0] not in got
    forced = llm.generate([p], SamplingParams(max_tokens=3, logit_bias={123: 1e4}))[0]
    assert forced.output_token_ids == [123] * 3
    for bad in (dict(allowed_token_ids=[512]), dict(allowed_token_ids=[]),
                dict(logit_bias={-1: 1.0})):
        with pytest.raises(ValueError):
            llm.generate([p], SamplingParams(max_tokens=2, **bad))


def test_min_tokens_masks_stop_tokens():
    """vLLM's ``min_tokens``: the stop tokens cannot be sampled until that
    many output tokens exist (a dense reference that masks them agrees), and
    the first stop after that ends the request."""
    from ._llama_ref import llama_logits

    llm = _llm()
    p = _prompts()[0]
    plain = llm.generate([p], SamplingParams(max_tokens=12, ignore_eos=True))[0].output_token_ids
    stop = plain[0]
    sp = SamplingParams(max_tokens=12, stop_token_ids=[stop], min_tokens=4)
    got = llm.generate([p, p], [sp, SamplingParams(max_tokens=12, ignore_eos=True)])
    ids, want = p.clone(), []
    for i in range(12):
        lg = llama_logits(llm.model, ids)[-1].clone()
        if i < 4:
            lg[stop] = float("-inf")
        t = int(lg.argmax())
        want.append(t)
        ids = torch.cat([ids, torch.tensor([t])])
        if t == stop:
            break
    assert got[0].output_token_ids == want and stop not in want[:4]
    assert got[1].output_token_ids == plain


def test_bad_words_match_dense_reference():
    """vLLM's ``bad_words``: the last token of a word is banned whenever the
    output ends with the rest of it (a one-token word is banned outright);
    greedy tokens equal a dense reference applying that rule."""
    from ._llama_ref import llama_logits

    class CsvTok:  # "5,9" -> [5, 9]
        def encode(self, text, add_special_tokens=False):
            return [int(x) for x in text.strip().split(",") if x]

        def decode(self, ids, skip_special_tokens=True):
            return ",".join(map(str, ids))

    llm = _llm()
    llm.set_tokenizer(CsvTok())
    p = _prompts()[2]
    plain = llm.generate([p], SamplingParams(max_tokens=12, ignore_eos=True))[0].output_token_ids
    words = [[plain[2]], [plain[4], plain[5]], [plain[0], plain[1], plain[6]]]
    sp = SamplingParams(max_tokens=12, ignore_eos=True,
                        bad_words=[",".join(map(str, w)) for w in words])
    got = llm.generate([p, p], [sp, SamplingParams(max_tokens=12, ignore_eos=True)])
    ids, want = p.clone(), []
    for _ in range(12):
        lg = llama_logits(llm.model, ids)[-1].clone()
        for w in words:
            if len(w) - 1 <= len(want) and (len(w) == 1 or want[-(len(w) - 1):] == w[:-1]):
                lg[w[-1]] = float("-inf")
        t = int(lg.argmax())
        want.append(t)
        ids = torch.cat([ids, torch.tensor([t])])
    assert got[0].output_token_ids == want and plain[2] not in want and want != plain
    assert got[1].output_token_ids == plain
