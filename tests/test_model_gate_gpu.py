"""Model-level gate stand-in on the GPU: the small seeded Llama of tests/tiny_llama.py (pinned on the CPU to
the reference's own model) with B200Backend swapped in, as an unmodified engine would swap it.

- fp32 pools: greedy generation through ragged paged steps (scattered blocks, pools pre-filled with junk,
  chunked prefill) gives exactly the dense greedy tokens (the reference's tests/test_paged.py:136-146).
- bf16: the reference's G1b check (src/minillm/correctness.py:57-95, driven as tests/test_kernels.py:75-114
  drives it): teacher-forced ragged steps (one batched prefill of ragged prompts, then 24 decode steps) on
  the same GPU and model.  G1b calibrates its tolerance from a trusted implementation's own spread; here the
  truth is the reference's torch algorithm with attention in fp32, the noise is the same algorithm run the
  way the reference runs it (SDPA in the pool dtype, bf16), and B200Backend's drift from the truth (mean
  KL, max |delta logit|) must be within twice that noise (with G1b's floors), with top-1 agreement
  wherever the truth's lead is clear.  (Checked against itself, as test_kernels.py does for Llama-3.1-8B,
  only the floors would apply; they are calibrated for that model's sharp logits, not for a random one.)  The
  prefill rows of >= 16 tokens run as tensor-core query tiles; a second case has every row behind a shared
  24-block prefix, so the decode steps run the shared-prefix (cascade) kernel.
"""

from __future__ import annotations

import random

import pytest
import torch

from tiny_llama import (TinyConfig, TinyLlama, TorchPagedBackend, drift, g1b_passed, make_weights, prompt, run_paged,
                        teacher_forced)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def weights():
    return make_weights(TinyConfig())


def test_fp32_ragged_generation_matches_dense(mlb, cuda, weights):
    cfg = TinyConfig()
    cpu, gpu = TinyLlama(cfg, weights, "cpu"), TinyLlama(cfg, weights, cuda)
    ps = [prompt(1, 3), prompt(2, 17), prompt(3, 1), prompt(4, 40)]  # 40 tokens span three blocks
    got = run_paged(mlb, gpu, mlb.B200Backend(check_errors=True), ps, 20)
    assert got == [cpu.greedy_dense(p, 20) for p in ps]


def test_fp32_chunked_prefill_matches_dense(mlb, cuda, weights):
    cfg = TinyConfig()
    cpu, gpu = TinyLlama(cfg, weights, "cpu"), TinyLlama(cfg, weights, cuda)
    ps = [prompt(5, 30), prompt(6, 21)]
    got = run_paged(mlb, gpu, mlb.B200Backend(check_errors=True), ps, 8, chunk_first=13)
    assert got == [cpu.greedy_dense(p, 8) for p in ps]


class _Recording:
    """B200Backend that records, per forward, whether the plan held query tiles / shared-prefix units and
    whether the append rode in the attention launch."""

    def __init__(self, mlb):
        self.inner = mlb.B200Backend(check_errors=True)
        self.seen = set()

    def forward(self, q, k, v, k_cache, v_cache, meta):
        out = self.inner.forward(q, k, v, k_cache, v_cache, meta)
        p = self.inner._plan
        if p.has_query_tiles:
            self.seen.add("query_tiles")
        if p.num_shared_units and not p.has_query_tiles:
            self.seen.add("shared_prefix")
        if self.inner.last_append_fused:
            self.seen.add("fused_append")
        return out


@pytest.mark.parametrize("shared", [0, 24], ids=["ragged", "shared_prefix"])
def test_bf16_teacher_forced_drift_within_g1b(mlb, cuda, weights, shared):
    cfg = TinyConfig()
    model = TinyLlama(cfg, weights, cuda, torch.bfloat16)
    rng = random.Random(0)
    head = [rng.randrange(cfg.vocab_size) for _ in range(shared * 16)]
    lens = (12, 200, 57, 1, 640, 33, 90, 8)
    seqs = [head + [rng.randrange(cfg.vocab_size) for _ in range(n + 24)] for n in lens]
    prompt_lens = [len(s) - 24 for s in seqs]
    truth = teacher_forced(mlb, model, TorchPagedBackend(torch.float32), seqs, prompt_lens, 24, shared=shared)
    ref_bf16 = teacher_forced(mlb, model, TorchPagedBackend(), seqs, prompt_lens, 24, shared=shared)
    ours_backend = _Recording(mlb)
    ours = teacher_forced(mlb, model, ours_backend, seqs, prompt_lens, 24, shared=shared)
    noise, got = drift(truth, ref_bf16), drift(truth, ours)
    print(f"\nG1b tiny llama bf16 ({'shared prefix' if shared else 'ragged'}): ours {got}, noise {noise}")
    assert g1b_passed(noise, got), (got, noise)
    assert "fused_append" in ours_backend.seen
    assert "query_tiles" in ours_backend.seen  # the prefill rows of >= 16 tokens
    if shared:
        assert "shared_prefix" in ours_backend.seen
