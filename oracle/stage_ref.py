"""CPU restatement of one pipeline stage and of the pipeline coordinator.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Every function cites the
reference code it restates.  Rounding points follow the reference: each
PyTorch op on a bf16 tensor returns bf16, so an elementwise chain rounds after
every op, while matmuls accumulate in fp32 and round once.

``cfg`` is any object with the LlamaConfig fields (vocab_size, hidden_size,
intermediate_size, num_hidden_layers, num_attention_heads,
num_key_value_heads, head_dim, max_position_embeddings, rms_norm_eps,
rope_theta) plus ``qk_norm`` / ``mask_policy`` / ``attention_implementation``
when present.  State dicts use the reference stage's key names.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

KV = list  # list[(k, v)] per local layer, each [B, nkv, T, D]


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm.forward (models/llama_dense.py:91-93); HF Qwen3RMSNorm is the same."""
    r = x.float().pow(2).mean(-1, keepdim=True).add(eps).rsqrt()
    return (x.float() * r).to(x.dtype) * w


def rope_tables(cfg, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """_precompute_freqs (llama_dense.py:96-104) cast as at :431-432.

    HF Qwen3 stages (mask_policy "cache") hold the inverse frequencies as a
    buffer that Qwen3Stage's ``self.to(dtype)`` rounds to the stage dtype
    (qwen3_hf.py:139-140); Qwen3RotaryEmbedding.forward then forms the angles
    from them in fp32 and casts cos/sin to the activation dtype."""
    dim = cfg.head_dim
    freqs = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2).float() / dim))
    if getattr(cfg, "mask_policy", "llama") == "cache":
        freqs = freqs.to(dtype).float()
    t = torch.arange(cfg.max_position_embeddings).float()
    f = torch.outer(t, freqs)
    return f.cos().to(dtype), f.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """_rotate_half + _apply_rope (llama_dense.py:107-125); x [B, h, S, D]."""
    c = torch.cat([cos, cos], dim=-1)[pos].unsqueeze(1)
    s = torch.cat([sin, sin], dim=-1)[pos].unsqueeze(1)
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return (x * c) + (rot * s)


def visible_mask(cfg, B: int, S: int, past: int, pos: torch.Tensor) -> torch.Tensor | None:
    """Boolean [B, S, past+S] visibility, or None when every key is visible.

    LlamaStage mask policy (llama_dense.py:497-532): sdpa with S == 1 uses no
    mask; otherwise key j is visible iff j <= position.  HF's Qwen3 causal mask
    (qwen3_hf.py:232-245 -> transformers create_causal_mask) uses the cache
    index: j <= past + s.
    """
    keys = torch.arange(past + S)
    if getattr(cfg, "mask_policy", "llama") == "cache":
        q = torch.arange(past, past + S).view(1, S, 1).expand(B, S, 1)
        return keys.view(1, 1, -1) <= q
    if getattr(cfg, "attention_implementation", "sdpa") == "sdpa" and S == 1:
        return None
    return keys.view(1, 1, -1) <= pos.view(B, S, 1)


def attention(cfg, q, k, v, allowed) -> torch.Tensor:
    """Grouped-query attention with scale 1/sqrt(D).

    sdpa path (llama_dense.py:173-215): softmax(q k^T * scale) v in fp32,
    output rounded to the activation dtype.  eager path (:216-227): scores
    rounded to the dtype, divided by sqrt(D), softmax in fp32 cast back.
    q [B, nq, S, D]; k, v [B, nkv, T, D]; allowed [B, S, T] or None.
    """
    nq, nkv, D = q.shape[1], k.shape[1], q.shape[-1]
    g = nq // nkv
    kk = k.repeat_interleave(g, dim=1)
    vv = v.repeat_interleave(g, dim=1)
    if getattr(cfg, "attention_implementation", "sdpa") == "eager" and getattr(cfg, "mask_policy", "llama") != "cache":
        scores = torch.matmul(q, kk.transpose(2, 3)) / math.sqrt(D)
        if allowed is not None:
            scores = scores.masked_fill(~allowed.unsqueeze(1), torch.finfo(q.dtype).min)
        p = torch.softmax(scores.float(), dim=-1).to(q.dtype)
        return torch.matmul(p, vv)
    acc = torch.float64 if _EXACT[-1] else torch.float32
    scores = torch.matmul(q.to(acc), kk.to(acc).transpose(2, 3)) * (1.0 / math.sqrt(D))
    if allowed is not None:
        scores = scores.masked_fill(~allowed.unsqueeze(1), float("-inf"))
    p = torch.softmax(scores, dim=-1)
    return torch.matmul(p, vv.to(acc)).to(q.dtype)


_EXACT = [False]


class exact_rounding:
    """Within this context the oracle accumulates matmuls and attention in
    float64 and rounds once to the activation dtype at the reference's
    rounding points: the exactly-rounded computation that any fp32 or bf16
    implementation (the reference's CPU path included) approximates."""

    def __enter__(self):
        _EXACT.append(True)
        return self

    def __exit__(self, *exc):
        _EXACT.pop()


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """nn.Linear without bias (llama_dense.py:140-143, 239-241)."""
    if _EXACT[-1]:
        return torch.nn.functional.linear(x.double(), w.double()).to(x.dtype)
    return torch.nn.functional.linear(x, w)


def decoder_layer(cfg, sd: dict, p: str, x, cos, sin, pos, cache, allowed):
    """LlamaDecoderLayer.forward (llama_dense.py:259-281) with GQAttention
    (:145-229); with qk_norm, HF Qwen3Attention's q_norm/k_norm before RoPE."""
    B, S, _ = x.shape
    nq, nkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    eps = cfg.rms_norm_eps
    h = rms_norm(x, sd[p + "input_layernorm.weight"], eps)
    q = linear(h, sd[p + "self_attn.q_proj.weight"]).view(B, S, nq, D)
    k = linear(h, sd[p + "self_attn.k_proj.weight"]).view(B, S, nkv, D)
    v = linear(h, sd[p + "self_attn.v_proj.weight"]).view(B, S, nkv, D)
    if getattr(cfg, "qk_norm", False):
        q = rms_norm(q, sd[p + "self_attn.q_norm.weight"], eps)
        k = rms_norm(k, sd[p + "self_attn.k_norm.weight"], eps)
    q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    q = apply_rope(q, cos, sin, pos)
    k = apply_rope(k, cos, sin, pos)
    if cache is not None:
        k = torch.cat([cache[0], k], dim=2)
        v = torch.cat([cache[1], v], dim=2)
    a = attention(cfg, q, k, v, allowed)
    a = a.transpose(1, 2).reshape(B, S, nq * D)
    x = x + linear(a, sd[p + "self_attn.o_proj.weight"])
    h = rms_norm(x, sd[p + "post_attention_layernorm.weight"], eps)
    gate = linear(h, sd[p + "mlp.gate_proj.weight"])
    up = linear(h, sd[p + "mlp.up_proj.weight"])
    x = x + linear(torch.nn.functional.silu(gate) * up, sd[p + "mlp.down_proj.weight"])
    return x, (k, v)


@dataclass
class OracleStage:
    """LlamaStage (llama_dense.py:293-578) / Qwen3Stage restated on the CPU."""

    cfg: object
    layer_start: int
    layer_end: int
    has_embedding: bool
    has_lm_head: bool
    state: dict
    dtype: torch.dtype = torch.float32
    caches: dict = field(default_factory=dict)

    def __post_init__(self):
        self.state = {k: v.detach().to("cpu", self.dtype) for k, v in self.state.items()}
        self.cos, self.sin = rope_tables(self.cfg, self.dtype)

    def cache_length(self, key=None) -> int:
        c = self.caches.get(key)
        return 0 if not c else int(c[0][0].shape[2])

    def forward(self, x=None, *, input_ids=None, position_ids=None, key=None, use_cache=True,
                last_only=False):
        """``last_only`` applies the final norm and lm_head to the last position
        only (the prefill logits a sampler reads); the layers see every position."""
        cfg = self.cfg
        if self.has_embedding:
            B, S = input_ids.shape
            x = self.state["embed_tokens.weight"][input_ids.long()]
        else:
            x = x.to("cpu", self.dtype)
            B, S = x.shape[0], x.shape[1]
        cache = self.caches.get(key) if use_cache else None
        past = 0 if not cache else int(cache[0][0].shape[2])
        if position_ids is None:
            pos = torch.arange(past, past + S).unsqueeze(0).expand(B, -1)
        else:
            pos = position_ids.to("cpu").long().expand(B, S)
        allowed = visible_mask(cfg, B, S, past, pos)
        new = []
        for i in range(self.layer_end - self.layer_start):
            x, kv = decoder_layer(
                cfg, self.state, f"layers.{i}.", x, self.cos, self.sin, pos,
                cache[i] if cache else None, allowed,
            )
            new.append(kv)
        if use_cache:
            self.caches[key] = new
        if self.has_lm_head:
            if last_only:
                x = x[:, -1:]
            x = linear(rms_norm(x, self.state["norm.weight"], cfg.rms_norm_eps), self.state["lm_head.weight"])
        return x

    def trim(self, length: int, key=None) -> None:
        c = self.caches.get(key)
        if not c:
            return
        self.caches[key] = [(k[:, :, :length], v[:, :, :length]) for k, v in c]

    def clear(self, key=None) -> None:
        self.caches.pop(key, None)


def split_layers(n_layers: int, n_stages: int) -> list[tuple[int, int]]:
    """build_pipeline's even split (backends/portable/pipeline.py:67-74)."""
    base, rem = divmod(n_layers, n_stages)
    out, start = [], 0
    for i in range(n_stages):
        end = start + base + (1 if i < rem else 0)
        out.append((start, end))
        start = end
    return out


def build_stages(cfg, n_stages: int, full_state: dict, dtype=torch.float32, ranges=None) -> list[OracleStage]:
    """One OracleStage per range, weights cut from a whole-model state dict."""
    ranges = ranges or split_layers(cfg.num_hidden_layers, n_stages)
    stages = []
    for i, (a, b) in enumerate(ranges):
        sd = {}
        for g in range(a, b):
            pre = f"layers.{g}."
            for k, v in full_state.items():
                if k.startswith(pre):
                    sd[f"layers.{g - a}." + k[len(pre):]] = v
        first, last = i == 0, i == len(ranges) - 1
        if first:
            sd["embed_tokens.weight"] = full_state["embed_tokens.weight"]
        if last:
            sd["norm.weight"] = full_state["norm.weight"]
            sd["lm_head.weight"] = full_state.get("lm_head.weight", full_state["embed_tokens.weight"])
        stages.append(OracleStage(cfg, a, b, first, last, sd, dtype))
    return stages


def prefill(stages: list[OracleStage], input_ids: torch.Tensor, key=None, last_only=False) -> torch.Tensor:
    """pipeline_prefill (pipeline.py:110-163): clear, then stages in order."""
    for s in stages:
        s.clear(key)
    h = None
    for i, s in enumerate(stages):
        h = s.forward(h, input_ids=input_ids if i == 0 else None, key=key, last_only=last_only)
    return h


def decode_step(stages: list[OracleStage], next_token: torch.Tensor, key=None) -> torch.Tensor:
    """pipeline_decode_step (pipeline.py:166-233): positions arange(T, T+S)."""
    B, S = next_token.shape
    T = stages[0].cache_length(key)
    pos = torch.arange(T, T + S).unsqueeze(0).expand(B, -1)
    h = None
    for i, s in enumerate(stages):
        h = s.forward(h, input_ids=next_token if i == 0 else None, position_ids=pos, key=key)
    return h


def greedy(logits: torch.Tensor) -> torch.Tensor:
    """greedy_sample (sampling.py:58-60): argmax, first index on ties."""
    return logits.argmax(dim=-1)


def top_p_nucleus(logits: torch.Tensor, temperature: float, top_p: float):
    """The distribution top_p_sample hands to multinomial (sampling.py:82-92).

    Returns (sorted_probs renormalised [rows, V], sorted_indices [rows, V]);
    ties are ordered by token index (a stable sort).
    """
    probs = torch.softmax(logits.float() / temperature, dim=-1)
    sp, si = torch.sort(probs, descending=True, dim=-1, stable=True)
    cum = torch.cumsum(sp, dim=-1)
    sp = sp.clone()
    sp[cum - sp > top_p] = 0.0
    sp = sp / sp.sum(dim=-1, keepdim=True).clamp(min=1e-12)
    return sp, si


def top_p_with_uniforms(logits: torch.Tensor, temperature: float, top_p: float, u: torch.Tensor) -> torch.Tensor:
    """top_p_sample with the multinomial draw replaced by inverse-CDF sampling
    of a given uniform per row: the first sorted token whose cumulative
    renormalised probability exceeds u."""
    if temperature <= 0:
        return greedy(logits)
    flat = logits.reshape(-1, logits.shape[-1])
    sp, si = top_p_nucleus(flat, temperature, top_p)
    cum = torch.cumsum(sp, dim=-1)
    u = u.reshape(-1, 1).float()
    idx = (cum <= u).sum(dim=-1, keepdim=True).clamp(max=flat.shape[-1] - 1)
    # never land on a removed (zero-probability) token
    kept = (sp > 0).sum(dim=-1, keepdim=True) - 1
    idx = torch.minimum(idx, kept)
    return si.gather(-1, idx).squeeze(-1).reshape(logits.shape[:-1])


def top_p_acceptable(logits: torch.Tensor, temperature: float, top_p: float, u: float,
                     eps: float = 1e-5) -> set[int]:
    """Token ids a correct fp32 top-p sampler may return for uniform ``u``.

    The same algorithm as top_p_with_uniforms, in float64, with every
    boundary widened by ``eps``: tokens whose cumulative-probability interval
    comes within eps of u, for every kept-prefix length a sampler may reach
    when the exclusive masses within eps of top_p fall either side of the cut
    (each length renormalises differently).  One row of logits [V].
    """
    probs = torch.softmax(logits.double() / temperature, dim=-1)
    sp, si = torch.sort(probs, descending=True, stable=True)
    excl = torch.cumsum(sp, 0) - sp
    n_lo = max(1, int((excl <= top_p - eps).sum()))
    n_hi = max(1, int((excl <= top_p + eps).sum()))
    out: set[int] = set()
    for n in range(n_lo, n_hi + 1):
        kp = sp[:n] / sp[:n].sum()
        inc = torch.cumsum(kp, 0)
        exc = inc - kp
        hit = (inc > u - eps) & (exc <= u + eps)
        out.update(si[:n][hit].tolist())
    return out


def exact_bar(got: torch.Tensor, ref: torch.Tensor, exact: torch.Tensor, what: str = "") -> dict:
    """The bf16 parity bar at full model width, where north of 2e-2 max-abs is
    the reference's own rounding noise: the implementation under test must be
    no further from the exactly-rounded computation (``exact_rounding``) than
    the reference's bf16 arithmetic (this oracle, or the reference itself) is:

        mean |got - exact| <= 1.5 * mean |ref - exact| + 1e-3
        max  |got - exact| <= max(2e-2, 2 * max |ref - exact|)

    Raises AssertionError with the figures; returns them otherwise."""
    e_got, e_ref = (got.float() - exact.float()).abs(), (ref.float() - exact.float()).abs()
    stats = {
        "mean_got": float(e_got.mean()), "mean_ref": float(e_ref.mean()),
        "max_got": float(e_got.max()), "max_ref": float(e_ref.max()),
        "max_got_vs_ref": float((got.float() - ref.float()).abs().max()),
    }
    assert stats["mean_got"] <= 1.5 * stats["mean_ref"] + 1e-3, (what, stats)
    assert stats["max_got"] <= max(2e-2, 2 * stats["max_ref"]), (what, stats)
    return stats
