"""Oracle: one transformer pass over a paged cache. TEST INFRASTRUCTURE ONLY.

Restates kvengine/forward.py:147-215 (`forward_with_own_cache`) with the
HuggingFace Qwen2 module math spelled out (the reference calls those modules at
forward.py:176,180,191,194-196,204,207,212,215):

  hidden = embed[ids]
  per layer: h = rmsnorm(hidden); q,k,v = linear(h) (+bias); rope(q,k)
             (forward.py:55-69, rotate-half); k_all,v_all = cache.write(...)
             (paged.py:288-331); attn = attend(q, k_all, v_all, causal mask)
             (forward.py:85-144: repeat_kv, SDPA with an additive finfo.min
             mask, scale hd^-0.5); hidden += o_proj(attn)
             hidden += down(silu(gate(rmsnorm(hidden))) * up(...))
  cache.commit(T); logits = lm_head(rmsnorm(hidden)) (all rows or the last).

Works on a plain state dict under HuggingFace names (`kvengine_b200.weights`
produces one), in fp32 or bf16, on CPU.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


class OracleModel:
    """Weights + shapes. `roll_head` reproduces the reference tests' HostileDraft
    (tests/test_phase5.py:35-50: logits rolled by one along the vocab axis)."""

    def __init__(self, cfg, state_dict, dtype=torch.float32, roll_head: int = 0):
        self.cfg = cfg
        self.dtype = dtype
        self.sd = {k: v.to(device="cpu", dtype=dtype) for k, v in state_dict.items()}
        self.roll_head = roll_head
        hd = cfg.head_dim
        self.inv_freq = 1.0 / (
            cfg.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.int64).to(dtype=torch.float) / hd)
        )

    def as_fp32(self) -> "OracleModel":
        """The same weights (already rounded to this model's dtype) evaluated in
        fp32: the exact answer that a bf16 evaluation approximates."""
        return OracleModel(self.cfg, self.sd, torch.float32, self.roll_head)

    def rmsnorm(self, x, w):
        xf = x.to(torch.float32)
        var = xf.pow(2).mean(-1, keepdim=True)
        xf = xf * torch.rsqrt(var + self.cfg.rms_norm_eps)
        return w * xf.to(self.dtype)

    def rope(self, positions):
        freqs = positions.float()[:, None] * self.inv_freq[None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos().to(self.dtype), emb.sin().to(self.dtype)

    def lm_head(self, h):
        logits = F.linear(h, self.sd["lm_head.weight"])
        if self.roll_head:
            logits = logits.roll(shifts=self.roll_head, dims=-1)
        return logits


def _rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat([-x[..., half:], x[..., :half]], dim=-1)


def causal_mask(q_len: int, kv_len: int, dtype):
    """kvengine/forward.py:85-103: query i sits at kv_len - q_len + i."""
    if q_len == 1:
        return None
    q_pos = torch.arange(kv_len - q_len, kv_len).unsqueeze(1)
    k_pos = torch.arange(kv_len).unsqueeze(0)
    mask = torch.zeros(q_len, kv_len, dtype=dtype)
    mask.masked_fill_(k_pos > q_pos, torch.finfo(dtype).min)
    return mask[None, None]


def attend(q, k, v, mask, scale, n_rep, use_sdpa=True):
    """kvengine/forward.py:106-144. q [1,nq,T,hd]; k,v [1,nkv,kv,hd] -> [1,T,nq,hd]."""
    if n_rep > 1:
        b, h, t, d = k.shape
        k = k[:, :, None].expand(b, h, n_rep, t, d).reshape(b, h * n_rep, t, d)
        v = v[:, :, None].expand(b, h, n_rep, t, d).reshape(b, h * n_rep, t, d)
    if use_sdpa:
        out = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=scale)
        return out.transpose(1, 2).contiguous()
    scores = torch.matmul(q, k.transpose(2, 3)) * scale
    if mask is not None:
        scores = scores + mask
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(probs, v).transpose(1, 2).contiguous()


@torch.no_grad()
def oracle_forward(model: OracleModel, ids: list[int], cache, all_logits: bool = False,
                   use_sdpa: bool = True, hidden_out: list | None = None):
    """One pass over `ids` appending to `cache` (an OracleSeq). Returns logits
    [T, V] if all_logits else [1, V]. If `hidden_out` is a list, the final
    normed hidden rows are appended to it (debug aid)."""
    cfg, sd, dt = model.cfg, model.sd, model.dtype
    T = len(ids)
    start = cache.length
    cache.reserve(T)
    hidden = sd["model.embed_tokens.weight"][torch.tensor(ids, dtype=torch.long)][None]  # [1,T,H]
    cos, sin = model.rope(torch.arange(start, start + T))
    cos, sin = cos[None, None], sin[None, None]  # [1,1,T,hd]
    mask = causal_mask(T, start + T, dt)
    hd, nq, nkv = cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
    for l in range(cfg.num_layers):
        p = f"model.layers.{l}."
        residual = hidden
        h = model.rmsnorm(hidden, sd[p + "input_layernorm.weight"])
        q = F.linear(h, sd[p + "self_attn.q_proj.weight"], sd[p + "self_attn.q_proj.bias"])
        k = F.linear(h, sd[p + "self_attn.k_proj.weight"], sd[p + "self_attn.k_proj.bias"])
        v = F.linear(h, sd[p + "self_attn.v_proj.weight"], sd[p + "self_attn.v_proj.bias"])
        q = q.view(1, T, nq, hd).transpose(1, 2)
        k = k.view(1, T, nkv, hd).transpose(1, 2)
        v = v.view(1, T, nkv, hd).transpose(1, 2)
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        k_all, v_all = cache.write(l, k[0], v[0], start)
        out = attend(q, k_all[None], v_all[None], mask, cfg.scaling, nq // nkv, use_sdpa)
        hidden = residual + F.linear(out.reshape(1, T, -1), sd[p + "self_attn.o_proj.weight"])
        residual = hidden
        h = model.rmsnorm(hidden, sd[p + "post_attention_layernorm.weight"])
        g = F.linear(h, sd[p + "mlp.gate_proj.weight"])
        u = F.linear(h, sd[p + "mlp.up_proj.weight"])
        hidden = residual + F.linear(F.silu(g) * u, sd[p + "mlp.down_proj.weight"])
    cache.commit(T)
    hidden = model.rmsnorm(hidden, sd["model.norm.weight"])
    if not all_logits:
        hidden = hidden[:, -1:, :]
    if hidden_out is not None:
        hidden_out.append(hidden[0].clone())
    return model.lm_head(hidden)[0]


def state_dict_from_device(model) -> dict:
    """HuggingFace-named CPU state dict holding exactly the weights of a
    kvengine_b200 `Model` (undoes the device packing: stacked q/k/v rows,
    interleaved gate/up rows, fp32 bias and norm copies), so the oracle can run
    the same weights the GPU ran."""
    w, cfg, i = model.weights, model.cfg, model.cfg.intermediate_size
    dt = model.dtype
    sd = {"model.embed_tokens.weight": w.embed.cpu(), "model.norm.weight": w.norm.cpu().to(dt),
          "lm_head.weight": w.lm_head.cpu()}
    qs, ks = cfg.q_size, cfg.kv_size
    for li, lw in enumerate(w.layers):
        p = f"model.layers.{li}."
        qkv, b = lw["w_qkv"].cpu(), lw["b_qkv"].cpu().to(dt)
        for n, a, z in (("q", 0, qs), ("k", qs, qs + ks), ("v", qs + ks, qs + 2 * ks)):
            sd[p + f"self_attn.{n}_proj.weight"] = qkv[a:z]
            sd[p + f"self_attn.{n}_proj.bias"] = b[a:z]
        sd[p + "self_attn.o_proj.weight"] = lw["w_o"].cpu()
        gu = lw["w_gu"].cpu().view(i, 2, -1)
        sd[p + "mlp.gate_proj.weight"], sd[p + "mlp.up_proj.weight"] = gu[:, 0], gu[:, 1]
        sd[p + "mlp.down_proj.weight"] = lw["w_down"].cpu()
        sd[p + "input_layernorm.weight"] = lw["ln1"].cpu().to(dt)
        sd[p + "post_attention_layernorm.weight"] = lw["ln2"].cpu().to(dt)
    return sd
