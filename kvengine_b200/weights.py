"""Seeded random-init weights for Qwen2-architecture models, and the device layout.

The reference loads trained checkpoints through HuggingFace
(kvengine/loader.py:35-52). With no checkpoints available, every model here is
random-init: Linear and Embedding weights ~ N(0, 0.02) (HuggingFace's
`initializer_range` default), RMSNorm weights 1, Linear biases 0, tied
embedding and lm_head. `init_state_dict` returns tensors under HuggingFace's
Qwen2 state-dict names, so the same weights can be loaded into a
`transformers.Qwen2ForCausalLM` (that is how the golden fixtures are made with
the reference) or packed into the device layout by `DeviceWeights`.

Device layout (one entry per layer, all row-major, K contiguous):
  w_qkv  [q+2kv, H]  q_proj, k_proj, v_proj rows stacked; b_qkv [q+2kv] fp32
  w_o    [H, q]
  w_gu   [2I, H]     gate and up rows interleaved (row 2j = gate_j, 2j+1 = up_j)
                     so one GEMM tile holds both halves of every SwiGLU pair
  w_down [H, I]
  ln1, ln2 [H] fp32  (values already rounded to the model dtype)
plus embed [V, H], lm_head [V, H] (the same storage when tied), norm [H].
"""

from __future__ import annotations

import torch

from .config import ModelConfig


def _normal(shape, std, gen, device, dtype):
    t = torch.empty(shape, dtype=torch.float32, device=device)
    t.normal_(0.0, std, generator=gen)
    return t.to(dtype)


def init_state_dict(
    cfg: ModelConfig,
    seed: int,
    dtype: torch.dtype = torch.float32,
    device: str | torch.device = "cpu",
    std: float = 0.02,
    bias_std: float = 0.0,
    norm_jitter: float = 0.0,
) -> dict[str, torch.Tensor]:
    """Deterministic random-init weights under HuggingFace Qwen2 names.

    `bias_std` / `norm_jitter` > 0 give non-trivial biases and norm weights so
    tests can see a dropped bias or norm weight; the default reproduces
    HuggingFace's initialisation distribution (zero bias, unit norm).
    """
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    h, i = cfg.hidden_size, cfg.intermediate_size
    sd: dict[str, torch.Tensor] = {}
    sd["model.embed_tokens.weight"] = _normal((cfg.vocab_size, h), std, gen, device, dtype)

    def norm_w():
        w = torch.ones(h, dtype=torch.float32, device=device)
        if norm_jitter:
            w = w + _normal((h,), norm_jitter, gen, device, torch.float32)
        return w.to(dtype)

    def bias(n):
        if bias_std:
            return _normal((n,), bias_std, gen, device, dtype)
        return torch.zeros(n, dtype=dtype, device=device)

    for l in range(cfg.num_layers):
        p = f"model.layers.{l}."
        sd[p + "self_attn.q_proj.weight"] = _normal((cfg.q_size, h), std, gen, device, dtype)
        sd[p + "self_attn.q_proj.bias"] = bias(cfg.q_size)
        sd[p + "self_attn.k_proj.weight"] = _normal((cfg.kv_size, h), std, gen, device, dtype)
        sd[p + "self_attn.k_proj.bias"] = bias(cfg.kv_size)
        sd[p + "self_attn.v_proj.weight"] = _normal((cfg.kv_size, h), std, gen, device, dtype)
        sd[p + "self_attn.v_proj.bias"] = bias(cfg.kv_size)
        sd[p + "self_attn.o_proj.weight"] = _normal((h, cfg.q_size), std, gen, device, dtype)
        sd[p + "mlp.gate_proj.weight"] = _normal((i, h), std, gen, device, dtype)
        sd[p + "mlp.up_proj.weight"] = _normal((i, h), std, gen, device, dtype)
        sd[p + "mlp.down_proj.weight"] = _normal((h, i), std, gen, device, dtype)
        sd[p + "input_layernorm.weight"] = norm_w()
        sd[p + "post_attention_layernorm.weight"] = norm_w()
    sd["model.norm.weight"] = norm_w()
    if cfg.tie_word_embeddings:
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    else:
        sd["lm_head.weight"] = _normal((cfg.vocab_size, h), std, gen, device, dtype)
    return sd


def state_dict_from_hf(model) -> dict[str, torch.Tensor]:
    """Pull the Qwen2 weights out of a HuggingFace model (or a look-alike).

    Reads only the attributes the reference's forward touches
    (kvengine/forward.py:168-215): `.model.embed_tokens`, `.model.layers[i]`
    {input_layernorm, post_attention_layernorm, self_attn.{q,k,v,o}_proj,
    mlp.{gate,up,down}_proj}, `.model.norm`, and `.lm_head`.
    """
    inner = model.model
    sd = {"model.embed_tokens.weight": inner.embed_tokens.weight.detach()}
    for l, layer in enumerate(inner.layers):
        p = f"model.layers.{l}."
        a, m = layer.self_attn, layer.mlp
        for name in ("q_proj", "k_proj", "v_proj"):
            lin = getattr(a, name)
            sd[p + f"self_attn.{name}.weight"] = lin.weight.detach()
            b = lin.bias
            sd[p + f"self_attn.{name}.bias"] = (
                b.detach() if b is not None else torch.zeros(lin.weight.shape[0], dtype=lin.weight.dtype)
            )
        sd[p + "self_attn.o_proj.weight"] = a.o_proj.weight.detach()
        sd[p + "mlp.gate_proj.weight"] = m.gate_proj.weight.detach()
        sd[p + "mlp.up_proj.weight"] = m.up_proj.weight.detach()
        sd[p + "mlp.down_proj.weight"] = m.down_proj.weight.detach()
        sd[p + "input_layernorm.weight"] = layer.input_layernorm.weight.detach()
        sd[p + "post_attention_layernorm.weight"] = layer.post_attention_layernorm.weight.detach()
    sd["model.norm.weight"] = inner.norm.weight.detach()
    head = model.lm_head
    sd["lm_head.weight"] = head.weight.detach() if hasattr(head, "weight") else head._head.weight.detach()
    return sd


def rope_tables(cfg: ModelConfig, n_positions: int) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [n_positions, head_dim/2] in fp32, computed on the host.

    Same arithmetic as the rotary module the reference calls
    (kvengine/forward.py:180 -> transformers Qwen2RotaryEmbedding): inv_freq =
    1 / theta^(2i/hd) in fp32, angle = position * inv_freq (one fp32 product),
    cos/sin in fp32. Computing the table on the host with torch's CPU math
    makes the device tables bit-identical to the reference's.
    """
    hd = cfg.head_dim
    inv_freq = 1.0 / (
        cfg.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.int64).to(dtype=torch.float) / hd)
    )
    pos = torch.arange(n_positions, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    return freqs.cos().contiguous(), freqs.sin().contiguous()


class DeviceWeights:
    """Weights packed into the device layout described in the module docstring."""

    def __init__(self, cfg: ModelConfig, sd: dict[str, torch.Tensor], dtype: torch.dtype,
                 device: str | torch.device, roll_lm_head: int = 0):
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        dev = self.device

        def to(t):
            return t.to(device=dev, dtype=dtype).contiguous()

        def to_f32(t):
            # Round through the model dtype first so products match the reference.
            return t.to(dtype).to(device=dev, dtype=torch.float32).contiguous()

        self.embed = to(sd["model.embed_tokens.weight"])
        head = sd["lm_head.weight"]
        if roll_lm_head:
            # logits.roll(s, -1) == rows of the head rolled by s.
            head = head.roll(roll_lm_head, dims=0)
        if head.data_ptr() == sd["model.embed_tokens.weight"].data_ptr() and not roll_lm_head:
            self.lm_head = self.embed
        else:
            self.lm_head = to(head)
        self.norm = to_f32(sd["model.norm.weight"])
        self.layers = []
        i = cfg.intermediate_size
        for l in range(cfg.num_layers):
            p = f"model.layers.{l}."
            w_qkv = torch.cat([sd[p + f"self_attn.{n}_proj.weight"] for n in ("q", "k", "v")], 0)
            b_qkv = torch.cat([sd[p + f"self_attn.{n}_proj.bias"] for n in ("q", "k", "v")], 0)
            gate = sd[p + "mlp.gate_proj.weight"]
            up = sd[p + "mlp.up_proj.weight"]
            gu = torch.stack([gate, up], dim=1).reshape(2 * i, -1)
            self.layers.append({
                "w_qkv": to(w_qkv),
                "b_qkv": to_f32(b_qkv),
                "w_o": to(sd[p + "self_attn.o_proj.weight"]),
                "w_gu": to(gu),
                "w_down": to(sd[p + "mlp.down_proj.weight"]),
                "ln1": to_f32(sd[p + "input_layernorm.weight"]),
                "ln2": to_f32(sd[p + "post_attention_layernorm.weight"]),
            })
        self._rope_n = 0
        self.rope_cos = self.rope_sin = None
        self.ensure_rope(4096)

    def ensure_rope(self, n_positions: int) -> None:
        if n_positions <= self._rope_n:
            return
        n = max(n_positions, 2 * self._rope_n, 4096)
        cos, sin = rope_tables(self.cfg, n)
        self.rope_cos = cos.to(self.device)
        self.rope_sin = sin.to(self.device)
        self._rope_n = n

    def weight_bytes(self) -> int:
        """Bytes of weights one full forward streams (body + lm_head, no embedding)."""
        total = self.lm_head.numel() * self.lm_head.element_size()
        for L in self.layers:
            for key in ("w_qkv", "w_o", "w_gu", "w_down"):
                total += L[key].numel() * L[key].element_size()
        return total
