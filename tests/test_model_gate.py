"""CPU half of the model-level gate stand-in (tests/tiny_llama.py): the small Llama is the reference's model,
the torch paged backend is the reference's algorithm, and the ragged driver reproduces dense generation.

- With the reference's source tree at hand: the same weights loaded into the reference's LlamaForCausalLM
  give the same logits, dense and on one ragged paged step through the reference's own TorchRefBackend,
  PagedKVCache and AttentionMetadata (src/minillm/model/llama.py, attention/torch_ref.py).
- Always: TorchPagedBackend equals the oracle; greedy generation through ragged paged steps (scattered
  blocks, junk-filled pools, chunked prefill) equals dense greedy generation (tests/test_paged.py:136-146).
"""

from __future__ import annotations

import importlib
import sys

import pytest
import torch

import oracle
from conftest import reference_src
from tiny_llama import TinyConfig, TinyLlama, TorchPagedBackend, make_weights, new_pools, prompt, run_paged

REF = reference_src()
needs_reference = pytest.mark.skipif(REF is None, reason="the reference's source tree is not at hand")


def _reference_model(cfg: TinyConfig, weights):
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    rc = importlib.import_module("minillm.model.config")
    rl = importlib.import_module("minillm.model.llama")
    conf = rc.LlamaConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                          intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                          num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                          head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta)
    model = rl.LlamaForCausalLM(conf)
    model.load_state_dict(weights, strict=True)
    return model.eval()


@needs_reference
def test_tiny_llama_is_the_reference_model():
    cfg = TinyConfig()
    w = make_weights(cfg)
    ours = TinyLlama(cfg, w, "cpu")
    ref = _reference_model(cfg, w)
    ids = prompt(7, 45)
    with torch.inference_mode():
        want = ref(torch.tensor([ids]))[0]
    torch.testing.assert_close(ours.logits_dense(ids), want, atol=1e-4, rtol=0)
    # one ragged paged step of three sequences through the reference's own paged path
    meta_mod = importlib.import_module("minillm.attention.metadata")
    paged_mod = importlib.import_module("minillm.cache.paged")
    seqs = [(0, 21, [3, 9]), (0, 5, [4]), (0, 37, [1, 7, 11])]
    toks = [prompt(10 + i, n) for i, (_, n, _) in enumerate(seqs)]
    ids_t = torch.tensor([t for tok in toks for t in tok])
    rmeta = meta_mod.AttentionMetadata.build([meta_mod.SeqStep(c, n, b) for c, n, b in seqs], 16, "cpu")
    cache = paged_mod.PagedKVCache(ref.config, 16, "cpu", torch.float32)
    with torch.inference_mode():
        want = ref(ids_t[None], kv_cache=cache.step(rmeta), last_index=rmeta.logits_index)[:, 0]
    mlb = importlib.import_module("mini-llm-inference-server_b200")
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, n, b) for c, n, b in seqs], 16, "cpu")
    k_pools, v_pools = new_pools(cfg, 16, "cpu", torch.float32, fill=0.0)
    got = ours.logits_ragged(ids_t, meta, TorchPagedBackend(), k_pools, v_pools)
    torch.testing.assert_close(got, want, atol=1e-4, rtol=0)
    for a, b in zip(k_pools, cache.k):
        assert torch.equal(a, b)


def test_torch_paged_backend_is_the_oracle(mlb):
    g = torch.Generator().manual_seed(3)
    seqs = [(0, 37, [1, 2, 3]), (90, 1, [4, 5, 6, 7, 8, 9]), (40, 25, [10, 11, 12, 13, 14]), (300, 1, list(range(15, 34)))]
    n = sum(s[1] for s in seqs)
    q, k, v = (torch.randn(n, h, 64, generator=g) for h in (8, 2, 2))
    kp, vp = torch.randn(40, 16, 2, 64, generator=g), torch.randn(40, 16, 2, 64, generator=g)
    meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, m, b) for c, m, b in seqs], 16, "cpu")
    k1, v1, k2, v2 = kp.clone(), vp.clone(), kp.clone(), vp.clone()
    got = TorchPagedBackend().forward(q, k, v, k1, v1, meta)
    want = oracle.forward(q, k, v, k2, v2, oracle.build_metadata(seqs, 16))
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
    torch.testing.assert_close(got, want, atol=1e-5, rtol=0)


@pytest.mark.parametrize("chunk", [None, 13])
def test_ragged_paged_generation_matches_dense_on_cpu(mlb, chunk):
    cfg = TinyConfig()
    model = TinyLlama(cfg, make_weights(cfg), "cpu")
    ps = [prompt(1, 3), prompt(2, 17), prompt(4, 40)] if chunk is None else [prompt(5, 30), prompt(6, 21)]
    got = run_paged(mlb, model, TorchPagedBackend(), ps, 6, chunk_first=chunk)
    assert got == [model.greedy_dense(p, 6) for p in ps]
