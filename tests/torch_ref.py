"""Test-only third opinion: a plain PyTorch fp32 decoder forward over a
prepared directory, written from the Hugging Face modeling of the dense
families (RMSNorm, rotate-half RoPE, GQA causal attention, SwiGLU; optional
biases, qwen3's per-head q/k RMSNorm before RoPE, mistral's sliding window).
Cross-checks the C++ oracle; never shipped."""

from __future__ import annotations

import numpy as np
import torch


class TorchQwen2:
    def __init__(self, prepared, cfg: dict, device: str = "cpu"):
        self.cfg = cfg
        self.dev = device
        self.w = {}
        for name, unit in prepared.units.items():
            self.w[name] = torch.from_numpy(np.array(unit.f32())).to(device)
        hd = cfg["head_dim"]
        i = torch.arange(hd // 2, dtype=torch.float32)
        self.inv_freq = (cfg["rope_theta"] ** (-2.0 * i / hd)).to(device)

    def _norm(self, x, w):
        ms = (x * x).mean(-1, keepdim=True)
        return x * torch.rsqrt(ms + self.cfg["rms_eps"]) * w

    def _rope(self, x, pos):  # x [T, H, D]
        ang = pos[:, None].float() * self.inv_freq[None, :]
        c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
        h = x.shape[-1] // 2
        a, b = x[..., :h], x[..., h:]
        return torch.cat([a * c - b * s, b * c + a * s], -1)

    @torch.no_grad()
    def forward(self, tokens):
        """Full-sequence causal forward; returns logits of every position."""
        c = self.cfg
        T = len(tokens)
        ids = torch.tensor(tokens, device=self.dev)
        x = self.w["model.embed_tokens.weight"][ids]
        pos = torch.arange(T, device=self.dev)
        group = c["q_heads"] // c["kv_heads"]
        mask = torch.full((T, T), float("-inf"), device=self.dev).triu(1)
        if c.get("sliding_window"):
            # query t sees keys t - window + 1 .. t
            mask = mask + torch.full((T, T), float("-inf"), device=self.dev).tril(-c["sliding_window"])
        for l in range(c["num_layers"]):
            p = f"model.layers.{l}."
            h = self._norm(x, self.w[p + "input_layernorm.weight"])
            q = h @ self.w[p + "self_attn.q_proj.weight"].T + self.w.get(p + "self_attn.q_proj.bias", 0)
            k = h @ self.w[p + "self_attn.k_proj.weight"].T + self.w.get(p + "self_attn.k_proj.bias", 0)
            v = h @ self.w[p + "self_attn.v_proj.weight"].T + self.w.get(p + "self_attn.v_proj.bias", 0)
            q = q.view(T, c["q_heads"], c["head_dim"])
            k = k.view(T, c["kv_heads"], c["head_dim"])
            if p + "self_attn.q_norm.weight" in self.w:
                q = self._norm(q, self.w[p + "self_attn.q_norm.weight"])
            if p + "self_attn.k_norm.weight" in self.w:
                k = self._norm(k, self.w[p + "self_attn.k_norm.weight"])
            q = self._rope(q, pos)
            k = self._rope(k, pos)
            v = v.view(T, c["kv_heads"], c["head_dim"])
            k = k.repeat_interleave(group, 1)
            v = v.repeat_interleave(group, 1)
            att = torch.einsum("thd,shd->hts", q, k) / (c["head_dim"] ** 0.5) + mask
            o = torch.einsum("hts,shd->thd", att.softmax(-1), v).reshape(T, -1)
            o = o @ self.w[p + "self_attn.o_proj.weight"].T + self.w.get(p + "self_attn.o_proj.bias", 0)
            x = x + o
            h = self._norm(x, self.w[p + "post_attention_layernorm.weight"])
            g = h @ self.w[p + "mlp.gate_proj.weight"].T
            u = h @ self.w[p + "mlp.up_proj.weight"].T
            x = x + (torch.nn.functional.silu(g) * u) @ self.w[p + "mlp.down_proj.weight"].T
        x = self._norm(x, self.w["model.norm.weight"])
        head = self.w["model.embed_tokens.weight"] if c["tie_word_embeddings"] else self.w["lm_head.weight"]
        return x @ head.T


TorchDecoder = TorchQwen2
