"""Teacher-forced accuracy gates.

A gate compares the teacher-forced log-probabilities of a build under test
(``LLM.score``: log p(x[i+1] | x[:i+1]) over fixed token sequences) with a
reference, relative to an ENVELOPE: the same statistic between two runs that
are both correct but differ in legitimate ways (chunk size, batch layout,
graph vs eager, kernel partitioning). A run passes when

  mean |d|  <= mean_factor  * envelope.mean   (plus an absolute floor)
  max  |d|  <= max_factor   * envelope.max
  count(|d| > envelope.max) <= count_factor * envelope.count + count_slack

so a planted bug -- a RoPE position off by one, a KV slot off by one, an
expert output scaled by 1.01 -- fails it while summation-order noise does
not. Raw log-probabilities are scored (no sampling), so the gate is
deterministic.

    python -m vllm_sm70_b200.eval.teacher_forced --model /path/to/ckpt \\
        --prompts 8 --len 512 [--chunk-a 16384 --chunk-b 512]

prints the envelope between two chunkings of the same prompts on this
device (the noise floor a gate's factors multiply).

Reference parity: the teacher-forced envelope gates and mutation checks of
the reference's model tests (``sm70/tests/models/test_m5_flint_sm70.py``,
``sm70/scripts/m5_teacher_forced.py``,
``sm70/tests/models/m5_mutations/m5_mutation.py``).
"""
from __future__ import annotations

import argparse
import json
from dataclasses import asdict, dataclass

import torch


@dataclass
class Envelope:
    mean: float     # mean |d| over all scored positions
    max: float      # max |d|
    count: int      # positions with |d| above ``threshold``
    threshold: float
    n: int          # scored positions


def delta(a: list[torch.Tensor], b: list[torch.Tensor], threshold: float | None = None) -> Envelope:
    """|a - b| statistics over the concatenated per-prompt log-probabilities."""
    if len(a) != len(b) or any(x.shape != y.shape for x, y in zip(a, b)):
        raise ValueError("score lists differ in shape")
    d = torch.cat([(x.double() - y.double()).abs() for x, y in zip(a, b)])
    if d.numel() == 0:
        return Envelope(0.0, 0.0, 0, threshold or 0.0, 0)
    if torch.isnan(d).any():
        return Envelope(float("inf"), float("inf"), int(d.numel()), threshold or 0.0,
                        int(d.numel()))
    mx = float(d.max())
    thr = mx if threshold is None else threshold
    return Envelope(float(d.mean()), mx, int((d > thr).sum()), thr, int(d.numel()))


@dataclass
class GateResult:
    passed: bool
    observed: Envelope
    limits: dict


def gate(ref: list[torch.Tensor], test: list[torch.Tensor], envelope: Envelope,
         mean_factor: float = 4.0, max_factor: float = 4.0, count_factor: float = 2.0,
         count_slack: int = 2, floor: float = 1e-6) -> GateResult:
    """Pass / fail of ``test`` against ``ref`` given the legitimate
    ``envelope`` (``floor`` keeps an all-zero envelope from demanding
    bitwise equality)."""
    obs = delta(ref, test, threshold=max(envelope.max, floor))
    limits = {"mean": mean_factor * envelope.mean + floor,
              "max": max_factor * envelope.max + floor,
              "count": count_factor * envelope.count + count_slack}
    ok = obs.mean <= limits["mean"] and obs.max <= limits["max"] and obs.count <= limits["count"]
    return GateResult(bool(ok), obs, limits)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--load-format", default="dummy", choices=["dummy", "safetensors"])
    ap.add_argument("--prompts", type=int, default=8)
    ap.add_argument("--len", type=int, default=512)
    ap.add_argument("--chunk-a", type=int, default=16384)
    ap.add_argument("--chunk-b", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    from ..engine import LLM

    g = torch.Generator().manual_seed(args.seed)
    res = {}
    for name, chunk in (("a", args.chunk_a), ("b", args.chunk_b)):
        llm = LLM(args.model, load_format=args.load_format, max_num_seqs=4,
                  max_model_len=args.len + 16, max_num_batched_tokens=chunk, tune_gemm=False)
        vocab = llm.cfg.vocab_size
        if not res:
            prompts = [torch.randint(0, vocab, (args.len,), generator=g)
                       for _ in range(args.prompts)]
        res[name] = llm.score(prompts)
        llm.shutdown()
        del llm
    env = delta(res["a"], res["b"])
    print(json.dumps({"envelope": asdict(env), "chunk_a": args.chunk_a, "chunk_b": args.chunk_b}))


if __name__ == "__main__":
    main()
