"""Engine end to end on CPU (fp32 reference ops): scheduler, block manager,
chunked prefill, decode loop and greedy sampling vs an independent dense
torch Llama."""
import torch

from vllm_sm70_b200.engine import LLM, SamplingParams
from vllm_sm70_b200.engine.block_manager import _PyAllocator, build_prefill_meta
from vllm_sm70_b200.models.config import ModelConfig

from ._llama_ref import greedy_reference

TINY = ModelConfig(arch="llama", hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=2,
                   head_dim=32, intermediate_size=256, vocab_size=512, rope_theta=10000.0,
                   rms_eps=1e-5, max_position=512)


def _llm(**kw):
    args = dict(max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
                enforce_eager=True, max_num_batched_tokens=40)
    args.update(kw)
    llm = LLM(TINY, **args)
    # Scale weights up so greedy decisions are well separated in fp32.
    return llm


def test_greedy_matches_dense_reference():
    llm = _llm()
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (7, 33, 50, 16, 3)]
    outs = llm.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))
    assert len(outs) == 5
    for p, o in zip(prompts, outs):
        assert o.output_token_ids == greedy_reference(llm.model, p, 6)


def test_chunked_prefill_equals_single_chunk():
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (60, 90)]
    a = _llm(max_num_batched_tokens=16).generate(prompts, SamplingParams(max_tokens=4))
    b = _llm(max_num_batched_tokens=4096).generate(prompts, SamplingParams(max_tokens=4))
    assert [o.output_token_ids for o in a] == [o.output_token_ids for o in b]


def test_block_allocator_and_meta():
    al = _PyAllocator(10, 1)
    b = al.allocate(3)
    assert b.tolist() == [1, 2, 3]
    al.free(b)
    assert al.num_free() == 9
    bt = torch.tensor([[5, 2, 0], [7, 0, 0]], dtype=torch.int32)
    pos, slots = build_prefill_meta(bt, torch.tensor([14, 0]), torch.tensor([4, 2]), 8)
    assert pos.tolist() == [14, 15, 16, 17, 0, 1]
    # positions 14,15 live in row block 1 (id 2); 16,17 in row block 2 (id 0)
    assert slots.tolist() == [2 * 8 + 6, 2 * 8 + 7, 0, 1, 56, 57]


def test_qwen3_moe_tiny_generates_and_is_batch_invariant():
    from vllm_sm70_b200.models.config import ModelConfig

    cfg = ModelConfig(arch="qwen3_moe", hidden_size=128, num_layers=2, num_heads=4,
                      num_kv_heads=2, head_dim=32, intermediate_size=256, vocab_size=512,
                      rope_theta=10000.0, rms_eps=1e-6, max_position=512, qk_norm=True,
                      num_experts=8, top_k=2, moe_intermediate_size=64)
    llm = LLM(cfg, max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
              enforce_eager=True, max_num_batched_tokens=64)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (9, 30)]
    both = llm.generate(prompts, SamplingParams(max_tokens=5))
    solo = [llm.generate([p], SamplingParams(max_tokens=5))[0] for p in prompts]
    assert [o.output_token_ids for o in both] == [o.output_token_ids for o in solo]


def test_qwen3_next_tiny_hybrid_generates_batch_invariant():
    from vllm_sm70_b200.models.config import ModelConfig

    cfg = ModelConfig(arch="qwen3_next", hidden_size=128, num_layers=4, num_heads=4,
                      num_kv_heads=2, head_dim=64, intermediate_size=256, vocab_size=512,
                      rope_theta=10000.0, rms_eps=1e-6, max_position=512, qk_norm=True,
                      num_experts=8, top_k=2, moe_intermediate_size=64,
                      shared_expert_intermediate_size=64,
                      layer_types=("linear_attention",) * 3 + ("attention",),
                      linear_num_k_heads=2, linear_num_v_heads=4, linear_k_head_dim=64,
                      linear_v_head_dim=64, attn_output_gate=True, partial_rotary_factor=0.25)
    llm = LLM(cfg, max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
              enforce_eager=True, max_num_batched_tokens=24)
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (9, 30)]
    both = llm.generate(prompts, SamplingParams(max_tokens=4))
    solo = [llm.generate([p], SamplingParams(max_tokens=4))[0] for p in prompts]
    assert [o.output_token_ids for o in both] == [o.output_token_ids for o in solo]


def test_speculative_greedy_equals_plain_greedy():
    """With T = 0 the speculative path (MTP drafts + verify + rejection) must
    emit exactly the plain greedy tokens, whatever the drafts are."""
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (6, 21, 40)]
    sp = SamplingParams(max_tokens=9, ignore_eos=True)
    # Sharpen the LM head so greedy choices are not decided by fp32 rounding of
    # near-tied logits (verify and decode sum in different orders).
    a, b = _llm(), _llm(speculative_k=3, max_model_len=128)
    for m in (a.model, b.model):
        m.lm_head.mul_(200.0)
    plain = a.generate(prompts, sp)
    spec = b.generate(prompts, sp)
    assert [o.output_token_ids for o in spec] == [o.output_token_ids for o in plain]


def test_speculative_hybrid_greedy_equals_plain():
    """Same property on the hybrid model: the GDN states are rolled back to the
    last accepted token after every verify."""
    from vllm_sm70_b200.models.config import ModelConfig

    cfg = ModelConfig(arch="qwen3_next", hidden_size=128, num_layers=4, num_heads=4,
                      num_kv_heads=2, head_dim=64, intermediate_size=256, vocab_size=512,
                      rope_theta=10000.0, rms_eps=1e-6, max_position=512, qk_norm=True,
                      num_experts=8, top_k=2, moe_intermediate_size=64,
                      shared_expert_intermediate_size=64,
                      layer_types=("linear_attention",) * 3 + ("attention",),
                      linear_num_k_heads=2, linear_num_v_heads=4, linear_k_head_dim=64,
                      linear_v_head_dim=64, attn_output_gate=True, partial_rotary_factor=0.25)
    kw = dict(max_num_seqs=4, max_model_len=128, block_size=16, dtype=torch.float32,
              enforce_eager=True, max_num_batched_tokens=64)
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (7, 25)]
    sp = SamplingParams(max_tokens=7, ignore_eos=True)
    a, b = LLM(cfg, **kw), LLM(cfg, speculative_k=3, **kw)
    for m in (a.model, b.model):
        m.lm_head.mul_(200.0)
    plain = a.generate(prompts, sp)
    spec = b.generate(prompts, sp)
    assert [o.output_token_ids for o in spec] == [o.output_token_ids for o in plain]


def test_temperature_sampling_runs_and_is_seeded():
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (5, 12)]
    sp = SamplingParams(max_tokens=6, temperature=0.7, seed=123, ignore_eos=True)
    a = _llm().generate(prompts, sp)
    assert all(len(o.output_token_ids) == 6 for o in a)


def test_prefix_caching_reuses_blocks_and_matches():
    """Requests sharing a prompt prefix reuse its KV blocks (fewer prefilled
    tokens) and generate exactly what a cache-free engine generates; blocks
    held only by the cache are evicted when allocation runs short."""
    g = torch.Generator().manual_seed(5)
    prefix = torch.randint(0, 512, (50,), generator=g)
    prompts = [torch.cat([prefix, torch.randint(0, 512, (n,), generator=g)]) for n in (5, 9, 17)]
    sp = SamplingParams(max_tokens=5, ignore_eos=True)
    ref = _llm()
    want = [ref.generate([p], sp)[0].output_token_ids for p in prompts]
    llm = _llm(enable_prefix_caching=True)
    got = [llm.generate([p], sp)[0].output_token_ids for p in prompts]
    assert got == want
    pc = llm.prefix_cache
    assert pc.hits >= 2 * 3  # 3 full blocks of the 50-token prefix, reused twice
    # the cache's blocks stay allocated between generate calls
    assert all(llm.runner.alloc.block_refcount(b) == 1 for b in pc.entries.values())
    # whole prompt cached: the last token is still prefilled
    again = llm.generate([prompts[0]], sp)[0].output_token_ids
    assert again == want[0]
    # scarcity: a tiny KV pool forces eviction of cache-only blocks
    small = _llm(enable_prefix_caching=True, num_kv_blocks=9)
    outs = [small.generate([p], sp)[0].output_token_ids for p in prompts]
    assert outs == want


def test_prefix_cache_keys_chain():
    from vllm_sm70_b200.engine.prefix_cache import block_keys

    a = torch.arange(64)
    b = torch.cat([torch.arange(16, 32), torch.arange(16), torch.arange(32, 64)])
    ka, kb = block_keys(a, 16, 4), block_keys(b, 16, 4)
    # same tokens in block 2 and 3 but after a different prefix: different keys
    assert ka[0] != kb[0] and ka[2] != kb[2] and ka[3] != kb[3]
    assert block_keys(a, 16, 2) == ka[:2]


def test_prefix_cache_host_tier_restores_evicted_blocks():
    """A tiny device pool forces the shared prefix out; the host tier keeps a
    copy and a later request restores it (no re-prefill) with identical output."""
    from vllm_sm70_b200.engine.prefix_cache import HostKVTier, PrefixCache

    g = torch.Generator().manual_seed(9)
    prefix = torch.randint(0, 512, (48,), generator=g)
    a = torch.cat([prefix, torch.randint(0, 512, (6,), generator=g)])
    others = [torch.randint(0, 512, (60,), generator=g) for _ in range(3)]
    b = torch.cat([prefix, torch.randint(0, 512, (7,), generator=g)])
    sp = SamplingParams(max_tokens=4, ignore_eos=True)
    ref = _llm()
    want_b = ref.generate([b], sp)[0].output_token_ids
    llm = _llm(enable_prefix_caching=True, num_kv_blocks=7)
    host = HostKVTier(llm.runner.kv, 32)
    llm.prefix_cache = PrefixCache(llm.runner.alloc, llm.runner.block_size, host)
    for p in [a] + others:
        llm.generate([p], sp)
    assert host.saved > 0  # the prefix blocks were pushed out to the host tier
    got_b = llm.generate([b], sp)[0].output_token_ids
    assert host.restored >= 2 and got_b == want_b


def test_prefix_cache_disk_tier_survives_the_engine(tmp_path):
    """A second engine (same model, same cache directory) starts with the
    first one's prompt blocks: it restores them from disk instead of
    prefilling and generates exactly what a cache-free engine does. An engine
    of another model (other seed) lives in another namespace and finds
    nothing; damaged files are refused, not read."""
    g = torch.Generator().manual_seed(21)
    prefix = torch.randint(0, 512, (48,), generator=g)
    a = torch.cat([prefix, torch.randint(0, 512, (5,), generator=g)])
    b = torch.cat([prefix, torch.randint(0, 512, (9,), generator=g)])
    sp = SamplingParams(max_tokens=4, ignore_eos=True)
    want_b = _llm().generate([b], sp)[0].output_token_ids
    first = _llm(enable_prefix_caching=True, prefix_cache_dir=str(tmp_path))
    first.generate([a], sp)
    disk = first.prefix_cache.disk
    assert disk.saved == 3 and len(list(disk.dir.glob("*.kv"))) == 3
    second = _llm(enable_prefix_caching=True, prefix_cache_dir=str(tmp_path))
    assert second.prefix_cache.disk.dir == disk.dir
    assert second.generate([b], sp)[0].output_token_ids == want_b
    assert second.prefix_cache.disk.restored == 3 and second.prefix_cache.hits == 3
    other = _llm(enable_prefix_caching=True, prefix_cache_dir=str(tmp_path), seed=7)
    assert other.prefix_cache.disk.dir != disk.dir
    other.generate([b], sp)
    assert other.prefix_cache.disk.restored == 0
    # a truncated file is refused and the block is prefilled instead
    for f in disk.dir.glob("*.kv"):
        f.write_bytes(f.read_bytes()[:100])
    third = _llm(enable_prefix_caching=True, prefix_cache_dir=str(tmp_path))
    assert third.generate([b], sp)[0].output_token_ids == want_b
    assert third.prefix_cache.disk.restored == 0
    # ... and replaced by a good copy when the block is cached again
    fourth = _llm(enable_prefix_caching=True, prefix_cache_dir=str(tmp_path))
    assert fourth.generate([b], sp)[0].output_token_ids == want_b
    assert fourth.prefix_cache.disk.restored == 3


def test_continuous_batching_feed():
    """Requests fed while others decode join the running batch and give the
    same greedy tokens as a plain batch call; an unservable request (longer
    than max_model_len) finishes with an error while the rest are served; a
    closed feed ends the call once the running requests are done."""
    g = torch.Generator().manual_seed(0)
    P = [torch.randint(0, 512, (n,), generator=g) for n in (7, 33, 12, 20, 9)]
    llm = _llm()
    ref = [o.output_token_ids for o in llm.generate(P, SamplingParams(max_tokens=6))]
    sp = SamplingParams(max_tokens=6)
    plan = {0: [(0, P[0].tolist(), sp), (1, P[1].tolist(), sp)],
            2: [(2, P[2].tolist(), sp), (99, list(range(200)), sp)],   # 99: too long
            4: [(3, P[3].tolist(), sp), (4, P[4].tolist(), sp)]}
    calls = []

    def feed(block):
        calls.append(block)
        n = len(calls) - 1
        if not plan:
            return None  # closed: finish what runs
        return plan.pop(n, [])

    done = {}
    out = llm.generate([], feed=feed, on_finish=lambda o: done.__setitem__(o.request_id, o))
    assert out == []
    assert [done[i].output_token_ids for i in range(5)] == ref
    assert done[99].error and done[99].output_token_ids == []
    assert all(done[i].error is None for i in range(5))


def test_text_prompts_and_chat_with_tokenizer():
    """With a tokenizer, ``generate`` takes text prompts and fills
    ``RequestOutput.text``; ``chat`` applies the chat template; without one,
    text prompts are refused with a clear error."""
    import pytest

    class Tok:
        def encode(self, text):
            return [ord(c) % 500 + 1 for c in text]

        def decode(self, ids, skip_special_tokens=True):
            return "".join(chr(65 + i % 26) for i in ids)

        def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=True, **kw):
            return self.encode("".join(m["content"] for m in messages) + "|a:")

    sp = SamplingParams(max_tokens=4)
    llm = _llm(tokenizer=Tok())
    o = llm.generate(["hello there"], sp)[0]
    ids_o = llm.generate([Tok().encode("hello there")], sp)[0]
    assert o.output_token_ids == ids_o.output_token_ids and o.text == Tok().decode(o.output_token_ids)
    c = llm.chat([{"role": "user", "content": "hi"}], sp)[0]
    assert c.prompt_token_ids == Tok().encode("hi|a:") and len(c.text) == 4
    two = llm.chat([[{"role": "user", "content": "a"}], [{"role": "user", "content": "b"}]], sp)
    assert len(two) == 2
    with pytest.raises(ValueError, match="tokenizer"):
        _llm().generate(["text"], sp)


def test_online_prefill_interleaves_with_decode():
    """Online (feed) mode: a long prompt that arrives while another request
    decodes is prefilled one chunk per scheduler iteration, and the running
    request keeps producing tokens between those chunks; both results equal
    a plain batch call."""
    g = torch.Generator().manual_seed(3)
    short, long_ = torch.randint(0, 512, (8,), generator=g), torch.randint(0, 512, (100,), generator=g)
    llm = _llm(max_num_batched_tokens=16)
    want_s = llm.generate([short], SamplingParams(max_tokens=40))[0].output_token_ids
    want_l = llm.generate([long_], SamplingParams(max_tokens=4))[0].output_token_ids
    events, calls = [], []
    plan = {0: [(0, short.tolist(), SamplingParams(max_tokens=40))],
            3: [(1, long_.tolist(), SamplingParams(max_tokens=4))]}

    def feed(block):
        calls.append(1)
        if not plan:
            return None
        return plan.pop(len(calls) - 1, [])

    done = {}
    llm.generate([], feed=feed, stream_interval=2,
                 on_tokens=lambda rid, ids, fin: events.append((rid, len(ids))),
                 on_finish=lambda o: done.__setitem__(o.request_id, o.output_token_ids))
    assert done[0] == want_s and done[1] == want_l
    first_long = next(i for i, (rid, n) in enumerate(events) if rid == 1 and n)
    admitted_at = 3  # the long prompt arrived with the 4th feed call
    short_between = sum(1 for rid, n in events[:first_long] if rid == 0 and n)
    # 100 prompt tokens / 16 per chunk = 7 chunks; the short request decodes between them
    assert short_between >= admitted_at + 5, events[:first_long + 1]


def test_single_prompt_forms():
    """One prompt may be passed as a flat list of ids, a 1-D tensor row or
    inside a list; all give the same tokens."""
    llm = _llm()
    ids = list(range(30, 45))
    sp = SamplingParams(max_tokens=3)
    a = llm.generate(ids, sp)
    b = llm.generate([ids], sp)
    c = llm.generate(torch.tensor([ids]), sp)
    assert len(a) == 1 and a[0].output_token_ids == b[0].output_token_ids == c[0].output_token_ids


def test_stop_strings_and_min_tokens():
    """``stop`` strings cut tokens and text (the stop string kept only with
    ``include_stop_str_in_output``); ``min_tokens`` ignores stop tokens and
    strings that end earlier."""
    from vllm_sm70_b200.engine.llm import _cut_at_stop_string, _truncate_at_stop

    dec = lambda ids: "".join(chr(97 + i % 26) for i in ids)  # noqa: E731 - one char per id
    toks = [0, 1, 2, 3, 2, 3, 4]                             # "abcdcde"
    sp = SamplingParams(stop=["cd"])
    assert _cut_at_stop_string(toks, sp, dec) == ([0, 1, 2, 3], "ab")
    sp = SamplingParams(stop=["cd"], include_stop_str_in_output=True)
    assert _cut_at_stop_string(toks, sp, dec) == ([0, 1, 2, 3], "abcd")
    sp = SamplingParams(stop=["cd"], min_tokens=5)  # the first "cd" ends at token 4
    assert _cut_at_stop_string(toks, sp, dec) == ([0, 1, 2, 3, 2, 3], "abcd")
    assert _truncate_at_stop([5, 7, 5, 7], SamplingParams(stop_token_ids=[7], min_tokens=3)) == [5, 7, 5, 7]
    assert _truncate_at_stop([5, 7, 5, 7], SamplingParams(stop_token_ids=[7])) == [5, 7]

    class Tok:
        def encode(self, text):
            return [ord(c) - 96 for c in text]

        def decode(self, ids, skip_special_tokens=True):
            return "".join(chr(97 + i % 26) for i in ids)

    llm = _llm(tokenizer=Tok())
    full = llm.generate(["hello"], SamplingParams(max_tokens=8))[0]
    stop = full.text[2:4]
    cut = llm.generate(["hello"], SamplingParams(max_tokens=8, stop=[stop]))[0]
    assert cut.text == full.text[: full.text.find(stop)]
    assert cut.output_token_ids == full.output_token_ids[: len(cut.text) + len(stop)]


def test_vllm_style_outputs():
    """vLLM-style call and result shape: ``use_tqdm`` is accepted and
    ``outputs[0].token_ids`` mirrors ``output_token_ids``."""
    llm = _llm()
    o = llm.generate([list(range(20, 30))], SamplingParams(max_tokens=3), use_tqdm=False)[0]
    assert o.outputs[0].token_ids == o.output_token_ids and o.outputs[0].index == 0


def test_n_samples_offline():
    """``SamplingParams(n=3)``: one RequestOutput per prompt whose
    ``outputs`` holds the three samples (seeded: distinct, reproducible)."""
    llm = _llm()
    sp = SamplingParams(max_tokens=6, temperature=1.5, seed=11, n=3)
    prompts = [list(range(20, 30)), list(range(40, 47))]
    a = llm.generate(prompts, sp)
    b = llm.generate(prompts, sp)
    assert len(a) == 2 and [len(o.outputs) for o in a] == [3, 3]
    assert [[c.token_ids for c in o.outputs] for o in a] == [[c.token_ids for c in o.outputs] for o in b]
    assert len({tuple(c.token_ids) for c in a[0].outputs}) > 1
    assert [c.index for c in a[1].outputs] == [0, 1, 2] and a[1].request_id == 1


def test_n_samples_ids_and_streaming_guard():
    """n > 1: every sample reports its prompt's index; streaming callbacks
    (which take one index per stream) are refused instead of receiving flat
    sample indices."""
    import pytest

    llm = _llm()
    sp = SamplingParams(max_tokens=3, temperature=1.0, seed=5, n=2)
    outs = llm.generate([list(range(20, 30)), list(range(40, 47))], sp)
    assert [o.request_id for o in outs] == [0, 1]
    assert all(m.request_id == o.request_id for o in outs for m in (o.more or []))
    with pytest.raises(ValueError, match="n = 1"):
        llm.generate([list(range(20, 30))], sp, on_tokens=lambda *a: None)


def test_stop_token_retires_request_early(monkeypatch):
    """A request whose output reaches a stop token retires at the end of that
    decode burst instead of decoding on to ``max_tokens``: its tokens equal the
    full run cut after the stop, it runs at most one burst of decode steps
    past it, its slot is reused by waiting requests, and the outputs carry
    vLLM's finish reasons ("stop" with the token id, else "length")."""
    from vllm_sm70_b200.engine.llm import _truncate_at_stop

    llm = _llm()
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (9, 14, 5, 22, 11, 8)]
    full = llm.generate(prompts, SamplingParams(max_tokens=40, ignore_eos=True))
    assert all(o.outputs[0].finish_reason == "length" for o in full)
    assert full[0].outputs[0].stop_reason is None
    t0 = full[0].output_token_ids
    stop = t0[5]
    k = t0.index(stop)
    sp = SamplingParams(max_tokens=40, stop_token_ids=[stop])
    one = llm.generate([prompts[0]], sp)[0]
    assert one.output_token_ids == t0[: k + 1]
    assert one.finish_reason == "stop" and one.outputs[0].stop_reason == stop
    assert llm.last_stats.decode_steps <= 16  # one burst, not 39 steps
    # six requests on four slots: retired slots take the waiting prompts
    many = llm.generate(prompts, sp)
    for f, o in zip(full, many):
        assert o.output_token_ids == _truncate_at_stop(f.output_token_ids, sp)
        assert o.finish_reason == ("stop" if stop in f.output_token_ids else "length")
    # 0 turns the scan off: same tokens, every request decodes to max_tokens
    monkeypatch.setenv("VLLM_B200_STOP_CHECK_STEPS", "0")
    off = llm.generate([prompts[0]], sp)[0]
    assert off.output_token_ids == t0[: k + 1] and llm.last_stats.decode_steps == 39


def test_truncate_prompt_and_text_options():
    """``truncate_prompt_tokens`` serves the prompt's last k tokens (offline
    and online); ``detokenize=False`` leaves the text empty;
    ``skip_special_tokens`` reaches the tokenizer."""
    calls = []

    class Tok:
        def encode(self, text):
            return [ord(c) - 96 for c in text]

        def decode(self, ids, skip_special_tokens=True):
            calls.append(skip_special_tokens)
            return "".join(chr(97 + i % 26) for i in ids)

    llm = _llm(tokenizer=Tok())
    g = torch.Generator().manual_seed(9)
    p = torch.randint(0, 512, (40,), generator=g)
    sp = SamplingParams(max_tokens=4, ignore_eos=True)
    tail = llm.generate([p[-12:]], sp)[0]
    cut = llm.generate([p], SamplingParams(max_tokens=4, ignore_eos=True,
                                           truncate_prompt_tokens=12))[0]
    assert cut.output_token_ids == tail.output_token_ids and cut.prompt_token_ids == p[-12:].tolist()
    done = {}
    items = [[(0, p, SamplingParams(max_tokens=4, ignore_eos=True, truncate_prompt_tokens=12))]]
    llm.generate([], feed=lambda block: items.pop(0) if items else None,
                 on_finish=lambda o: done.__setitem__(o.request_id, o))
    assert done[0].output_token_ids == tail.output_token_ids
    assert llm.generate([p], SamplingParams(max_tokens=2, detokenize=False))[0].text is None
    calls.clear()
    llm.generate([p], SamplingParams(max_tokens=2, skip_special_tokens=False))
    assert calls and not any(calls)


def _dense_beam_search(model, prompt, W, n, eos, lp_pen=1.0):
    """Independent beam search on a dense forward (vLLM's scoring rule)."""
    from ._llama_ref import llama_logits

    def score(toks, cum):
        k = len(toks) - (1 if toks[-1] == eos else 0)
        return cum / (k ** lp_pen)

    beams, done = [(prompt.tolist(), 0.0)], []
    for _ in range(n):
        cands = []
        for toks, cum in beams:
            lg = llama_logits(model, torch.tensor(toks))[-1].double()
            lsm = lg - torch.logsumexp(lg, 0)
            v, i = lsm.topk(2 * W)
            for lp, t in zip(v.tolist(), i.tolist()):
                (done if t == eos else cands).append((toks + [t], cum + lp))
        beams = sorted(cands, key=lambda b: score(*b), reverse=True)[:W]
    return [b[0] for b in sorted(done + beams, key=lambda b: score(*b), reverse=True)[:W]]


def test_beam_search_matches_dense_reference():
    """``LLM.beam_search`` keeps the beams a dense-forward beam search keeps
    (same candidates, vLLM's length-normalised score), EOS-ended beams
    included; beam width 1 is greedy decoding."""
    from vllm_sm70_b200.engine import BeamSearchParams

    class Tok:
        eos_token_id = 7

        def encode(self, text):
            return [ord(c) - 96 for c in text]

        def decode(self, ids, skip_special_tokens=True):
            return "".join(chr(97 + i % 26) for i in ids)

    llm = _llm(tokenizer=Tok())
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (6, 11)]
    outs = llm.beam_search(prompts, BeamSearchParams(beam_width=3, max_tokens=5))
    for p, o in zip(prompts, outs):
        want = _dense_beam_search(llm.model, p, 3, 5, eos=7)
        assert [s.tokens for s in o.sequences] == want
        assert o.sequences[0].text == Tok().decode(want[0][p.numel():])
    one = llm.beam_search(prompts[:1], BeamSearchParams(beam_width=1, max_tokens=4,
                                                        ignore_eos=True))[0].sequences[0]
    greedy = llm.generate(prompts[:1], SamplingParams(max_tokens=4, ignore_eos=True))[0]
    assert one.tokens[prompts[0].numel():] == greedy.output_token_ids


def test_priority_scheduling_admits_low_values_first():
    """LLM(scheduling_policy="priority"): with one batch slot, requests are
    served lowest priority value first (arrival order on ties), with the
    same tokens as in arrival order; priority needs the policy."""
    import pytest

    order = []
    llm = _llm(max_num_seqs=1, scheduling_policy="priority")
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 512, (n,), generator=g) for n in (5, 9, 7, 4)]
    sp = SamplingParams(max_tokens=3, ignore_eos=True)
    fifo = llm.generate(prompts, sp)
    outs = llm.generate(prompts, sp, priority=[3, 1, 3, 0],
                        on_tokens=lambda i, ids, fin: fin and order.append(i))
    assert order == [3, 1, 0, 2]
    assert [o.output_token_ids for o in outs] == [o.output_token_ids for o in fifo]
    with pytest.raises(ValueError):
        _llm().generate(prompts, sp, priority=[0, 0, 0, 0])


def test_vllm_prompt_dicts():
    """vLLM's TokensPrompt / TextPrompt dicts are accepted, alone or in a list."""
    from vllm.inputs import TokensPrompt

    class Tok:
        def encode(self, text):
            return [ord(c) - 96 for c in text]

        def decode(self, ids, skip_special_tokens=True):
            return "".join(chr(97 + i % 26) for i in ids)

    llm = _llm(tokenizer=Tok())
    sp = SamplingParams(max_tokens=3, ignore_eos=True)
    ids = [5, 9, 14, 3]
    want = llm.generate([ids], sp)[0].output_token_ids
    assert llm.generate(TokensPrompt(prompt_token_ids=ids), sp)[0].output_token_ids == want
    both = llm.generate([{"prompt_token_ids": ids}, {"prompt": "eint"}], sp)
    assert both[0].output_token_ids == want and both[1].prompt_token_ids == [5, 9, 14, 20]
