"""A small seeded Llama for engine-level checks of the paged path (test infrastructure).

The reference's model-level gate (src/minillm/correctness.py:57-83, tests/test_kernels.py:75-114) needs the
real Llama-3.1-8B weights, which are not here.  The stand-in is the reference's own token-exactness check
(tests/test_paged.py:99-146, tests/test_prefix_cache.py:112-209) on a small random Llama: greedy generation
through ragged paged steps, with the attention backend swapped, must give the same tokens as dense
generation.  Head dim 64 (the reference's tiny fixture uses 16, which the kernels do not take).

`TinyLlama` holds its weights as plain tensors under the Hugging Face / reference parameter names, so the
same state dict loads into the reference's `LlamaForCausalLM` (src/minillm/model/llama.py) for the CPU pin
in test_model_gate.py.  Its arithmetic is the standard Llama decoder: RMSNorm in fp32 then cast, rotate-half
RoPE (theta 500000), grouped-query attention, SwiGLU MLP, pre-norm residuals, final norm, lm_head.
"""

from __future__ import annotations

import random
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class TinyConfig:
    vocab_size: int = 512
    hidden_size: int = 256
    intermediate_size: int = 512
    num_hidden_layers: int = 2
    num_attention_heads: int = 8
    num_key_value_heads: int = 2
    head_dim: int = 64
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0


def make_weights(cfg: TinyConfig, seed: int = 0) -> dict[str, torch.Tensor]:
    """Seeded fp32 weights, named as in Hugging Face's LlamaForCausalLM."""
    g = torch.Generator().manual_seed(seed)
    d, f, h, hkv, dh = cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim

    def w(*shape, std=0.08):
        return torch.randn(*shape, generator=g) * std

    sd = {"model.embed_tokens.weight": w(cfg.vocab_size, d, std=1.0), "model.norm.weight": 1.0 + w(d, std=0.1),
          "lm_head.weight": w(cfg.vocab_size, d)}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        sd.update({p + "input_layernorm.weight": 1.0 + w(d, std=0.1),
                   p + "post_attention_layernorm.weight": 1.0 + w(d, std=0.1),
                   p + "self_attn.q_proj.weight": w(h * dh, d), p + "self_attn.k_proj.weight": w(hkv * dh, d),
                   p + "self_attn.v_proj.weight": w(hkv * dh, d), p + "self_attn.o_proj.weight": w(d, h * dh),
                   p + "mlp.gate_proj.weight": w(f, d), p + "mlp.up_proj.weight": w(f, d),
                   p + "mlp.down_proj.weight": w(d, f)})
    return sd


def prompt(seed: int, n: int, vocab: int = 512) -> list[int]:
    r = random.Random(seed)
    return [r.randrange(vocab) for _ in range(n)]


class TinyLlama:
    def __init__(self, cfg: TinyConfig, weights: dict[str, torch.Tensor], device, dtype=torch.float32) -> None:
        self.cfg = cfg
        self.w = {k: v.to(device=device, dtype=dtype) for k, v in weights.items()}
        self.device, self.dtype = torch.device(device), dtype
        dh = cfg.head_dim
        self.inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, dh, 2, dtype=torch.int64).float() / dh))

    def _norm(self, x, name):
        h = x.float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps)
        return self.w[name] * h.to(x.dtype)

    def _rope(self, x, positions):
        """x [T, heads, Dh] rotated at positions [T] (rotate-half pairing)."""
        ang = positions.float()[:, None].cpu() * self.inv_freq[None, :]
        emb = torch.cat([ang, ang], dim=-1).to(x.device)
        cos, sin = emb.cos().to(x.dtype)[:, None], emb.sin().to(x.dtype)[:, None]
        x1, x2 = x.chunk(2, dim=-1)
        return x * cos + torch.cat([-x2, x1], dim=-1) * sin

    def _layer(self, i, x, positions, attend):
        cfg, p = self.cfg, f"model.layers.{i}."
        t = x.shape[0]
        hx = self._norm(x, p + "input_layernorm.weight")
        q = (hx @ self.w[p + "self_attn.q_proj.weight"].T).view(t, cfg.num_attention_heads, cfg.head_dim)
        k = (hx @ self.w[p + "self_attn.k_proj.weight"].T).view(t, cfg.num_key_value_heads, cfg.head_dim)
        v = (hx @ self.w[p + "self_attn.v_proj.weight"].T).view(t, cfg.num_key_value_heads, cfg.head_dim)
        q, k = self._rope(q, positions), self._rope(k, positions)
        o = attend(i, q, k, v)  # [T, H, Dh]
        x = x + o.reshape(t, -1) @ self.w[p + "self_attn.o_proj.weight"].T
        hx = self._norm(x, p + "post_attention_layernorm.weight")
        mlp = F.silu(hx @ self.w[p + "mlp.gate_proj.weight"].T) * (hx @ self.w[p + "mlp.up_proj.weight"].T)
        return x + mlp @ self.w[p + "mlp.down_proj.weight"].T

    def logits_dense(self, ids: list[int]) -> torch.Tensor:
        """Causal attention over one whole sequence (no cache): logits [T, V] (the dense reference path)."""
        x = self.w["model.embed_tokens.weight"][torch.tensor(ids, device=self.device)]
        pos = torch.arange(len(ids))

        def attend(i, q, k, v):
            o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                               v.transpose(0, 1)[None], is_causal=True, enable_gqa=True)
            return o[0].transpose(0, 1)

        for i in range(self.cfg.num_hidden_layers):
            x = self._layer(i, x, pos, attend)
        return self._norm(x, "model.norm.weight") @ self.w["lm_head.weight"].T

    def greedy_dense(self, ids: list[int], steps: int) -> list[int]:
        ids, out = list(ids), []
        for _ in range(steps):
            nxt = int(self.logits_dense(ids)[-1].argmax())
            ids.append(nxt)
            out.append(nxt)
        return out

    def logits_ragged(self, ids: torch.Tensor, meta, backend, k_pools, v_pools) -> torch.Tensor:
        """One ragged paged step: ids [N] (every sequence's new tokens back to back), the backend's forward
        per layer on that layer's pools; logits [S, V] at each sequence's last new token."""
        x = self.w["model.embed_tokens.weight"][ids.to(self.device)]
        pos = meta.positions.to(torch.long)

        def attend(i, q, k, v):
            return backend.forward(q, k, v, k_pools[i], v_pools[i], meta)

        for i in range(self.cfg.num_hidden_layers):
            x = self._layer(i, x, pos, attend)
        last = meta.logits_index.to(self.device)
        return self._norm(x[last], "model.norm.weight") @ self.w["lm_head.weight"].T


class TorchPagedBackend:
    """The reference's torch backend restated for tensors on any device (test infrastructure): write the
    step's k/v at slot_mapping (paged_torch_ref.py:23-28), then per sequence gather its pages and run SDPA
    in the pool dtype with the causal mask aligned to the end of its context (paged_torch_ref.py:40-74)."""

    name = "torch_paged"

    def __init__(self, compute_dtype: torch.dtype | None = None) -> None:
        self.compute_dtype = compute_dtype  # None: SDPA in the pool dtype, as the reference runs it

    def forward(self, q, k, v, k_cache, v_cache, meta):
        bs = k_cache.shape[1]
        k_cache.view(-1, *k_cache.shape[2:]).index_copy_(0, meta.slot_mapping, k.to(k_cache.dtype))
        v_cache.view(-1, *v_cache.shape[2:]).index_copy_(0, meta.slot_mapping, v.to(v_cache.dtype))
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        qo, lens = meta.query_start_loc, meta.seq_lens
        tables = meta.block_tables.to(q.device)
        for s in range(len(lens)):
            a, b, length = qo[s], qo[s + 1], lens[s]
            n = b - a
            pages = -(-length // bs)
            dt = self.compute_dtype or k_cache.dtype
            kk = k_cache[tables[s, :pages]].reshape(-1, *k_cache.shape[2:])[:length].transpose(0, 1).to(dt)  # [Hkv, L, Dh]
            vv = v_cache[tables[s, :pages]].reshape(-1, *v_cache.shape[2:])[:length].transpose(0, 1).to(dt)
            mask = torch.ones(n, length, dtype=torch.bool, device=q.device).tril(diagonal=length - n)
            o = F.scaled_dot_product_attention(q[a:b].transpose(0, 1)[None].to(dt), kk[None], vv[None],
                                               attn_mask=mask, enable_gqa=True)
            out[a:b] = o[0].transpose(0, 1).to(q.dtype)
        return out


def new_pools(cfg: TinyConfig, num_blocks: int, device, dtype, fill: float | None = 1e4):
    """Per-layer K and V pools; filled with a large value so reading any slot a sequence does not own
    changes the logits (tests/test_paged.py:99-103's trick)."""
    shape = (num_blocks, 16, cfg.num_key_value_heads, cfg.head_dim)
    ks = [torch.full(shape, fill, device=device, dtype=dtype) for _ in range(cfg.num_hidden_layers)]
    vs = [torch.full(shape, fill, device=device, dtype=dtype) for _ in range(cfg.num_hidden_layers)]
    return ks, vs


def run_paged(mlb, model: TinyLlama, backend, prompts: list[list[int]], steps: int, chunk_first: int | None = None,
              num_blocks: int = 96, seed: int = 2) -> list[list[int]]:
    """Greedy generation of every prompt together, one ragged paged step per iteration: blocks handed out in
    a seeded random order, pools pre-filled with junk, an optional first prefill cut at `chunk_first`
    tokens (the rest of each prompt is prefilled on top of its own cached tokens)."""
    cfg = model.cfg
    k_pools, v_pools = new_pools(cfg, num_blocks, model.device, model.dtype)
    free = list(range(num_blocks))
    random.Random(seed).shuffle(free)
    tokens = [list(p) for p in prompts]
    blocks: list[list[int]] = [[] for _ in prompts]
    cached = [0] * len(prompts)
    gen: list[list[int]] = [[] for _ in prompts]
    while min(len(g) for g in gen) < steps:
        upto = [len(t) for t in tokens]
        if chunk_first and not any(cached):
            upto = [min(chunk_first, len(t)) for t in tokens]
        for i, b in enumerate(blocks):
            while len(b) * 16 < upto[i]:
                b.append(free.pop())
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(cached[i], upto[i] - cached[i], list(blocks[i]))
                                            for i in range(len(tokens))], 16, model.device)
        ids = torch.tensor([t for i, tok in enumerate(tokens) for t in tok[cached[i]:upto[i]]])
        logits = model.logits_ragged(ids, meta, backend, k_pools, v_pools)
        assert torch.isfinite(logits).all()
        nxt = logits.argmax(-1).tolist()
        for i in range(len(tokens)):
            if upto[i] < len(tokens[i]):  # a mid-prompt chunk: nothing sampled yet
                cached[i] = upto[i]
                continue
            cached[i] = len(tokens[i])
            tokens[i].append(nxt[i])
            gen[i].append(nxt[i])
    return gen


def teacher_forced(mlb, model: TinyLlama, backend, seqs: list[list[int]], prompt_lens: list[int], decode_steps: int,
                   shared: int = 0, num_blocks: int = 1024) -> list[torch.Tensor]:
    """The reference's G1b drive (tests/test_kernels.py:84-110) on the small model: one batched ragged prefill
    of the prompts, then `decode_steps` decode steps feeding each sequence's FIXED continuation; logits of
    every step [S, V] as float32 on the CPU.  With `shared` > 0 every sequence's first `shared` blocks are the
    same block ids (a prefix-cache hit; the sequences' first `shared` x 16 tokens must agree): a first step
    prefills them, and every sequence then starts on top of them."""
    cfg = model.cfg
    k_pools, v_pools = new_pools(cfg, num_blocks, model.device, model.dtype, fill=0.0)
    per = num_blocks // len(seqs)
    blocks = [list(range(i * per, (i + 1) * per)) for i in range(len(seqs))]
    if shared:
        for b in blocks[1:]:
            b[:shared] = blocks[0][:shared]
    out = []
    if shared:  # the shared prefix lands in the pool first, as an earlier request left it
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(0, shared * 16, blocks[0])], 16, model.device)
        model.logits_ragged(torch.tensor(seqs[0][:shared * 16]), meta, backend, k_pools, v_pools)
    cached = [shared * 16] * len(seqs)  # every sequence starts on top of the shared prefix (or of nothing)
    upto = list(prompt_lens)
    for _ in range(decode_steps + 1):
        meta = mlb.AttentionMetadata.build([mlb.SeqStep(c, u - c, b) for c, u, b in zip(cached, upto, blocks)], 16,
                                           model.device)
        ids = torch.tensor([t for s, c, u in zip(seqs, cached, upto) for t in s[c:u]])
        out.append(model.logits_ragged(ids, meta, backend, k_pools, v_pools).float().cpu())
        cached, upto = upto, [u + 1 for u in upto]
    return out


# The reference's G1b check (src/minillm/correctness.py:26-95), restated: drift of test logits from reference
# logits as the mean KL, the largest |delta logit| and the top-1 disagreements where the reference's top-1 /
# top-2 gap exceeds MARGIN; the limits are twice the noise, with floors.
KL_FLOOR, MAX_DIFF_FLOOR, MARGIN = 1e-5, 0.125, 0.5


def drift(reference: list[torch.Tensor], test: list[torch.Tensor]) -> dict:
    kls, max_diff, bad, n = [], 0.0, 0, 0
    for ref, tst in zip(reference, test):
        lp_ref, lp_tst = F.log_softmax(ref, -1), F.log_softmax(tst, -1)
        kls.append((lp_ref.exp() * (lp_ref - lp_tst)).sum(-1))
        max_diff = max(max_diff, (ref - tst).abs().max().item())
        top2 = ref.topk(2, dim=-1).values
        clear = (top2[:, 0] - top2[:, 1]) > MARGIN
        bad += int((clear & (ref.argmax(-1) != tst.argmax(-1))).sum())
        n += ref.shape[0]
    return {"mean_kl": torch.cat(kls).mean().item(), "max_abs_diff": max_diff, "top1_disagreements": bad,
            "positions": n}


def g1b_passed(noise: dict, ours: dict) -> bool:
    return (ours["mean_kl"] <= 2 * max(noise["mean_kl"], KL_FLOOR)
            and ours["max_abs_diff"] <= 2 * max(noise["max_abs_diff"], MAX_DIFF_FLOOR)
            and ours["top1_disagreements"] == 0)
