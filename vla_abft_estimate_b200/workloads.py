"""Model-level workloads of the protected path: random-init decoders whose
every projection is an ``nn.Linear``, so that ``AbftInjector``'s
``F.linear`` hook sees all of them.

* ``build_qwen2``: the Qwen2-7B-shaped decoder of the reference's model
  benchmark (pytorch/qwen_abft_benchmark.py:130-154 times Qwen2.5 prefill
  and decode through the hook). No checkpoint is available, so weights are
  random N(0, 0.02) at the published shapes: 28 layers, hidden 3584, 28
  query / 4 KV heads of 128, SwiGLU 18944, vocab 152064; QKV and gate+up
  are fused into one linear each (the GEMM shapes BASELINE lists).
* ``build_cogact``: a CogACT-style vision-language-action forward. The
  reference only enumerates its GEMM shapes analytically
  (cogact_estimate.py:126-359, COGACT_RESULTS.md:33-106); this module runs
  them: ViT-L/14 and SigLIP-So400m/14 encoders over 256 patches, an MLP
  projector, a Llama-2-7B-shaped decoder over 256 visual + 32 text tokens
  and a DiT-B action head (adaLN-zero blocks) denoising 16 action tokens of
  7 values over 10 steps.

Both take their shape dictionary as an argument, so tests can run the same
architecture at reduced depth.
"""
from __future__ import annotations

QWEN2_7B = dict(hidden=3584, inter=18944, layers=28, heads=28, kv_heads=4, head_dim=128, vocab=152064,
                rope_theta=1000000.0, eps=1e-6)


def build_qwen2(cfg, device, seed=0, dtype=None):
    """Qwen2-style decoder: RMSNorm, fused QKV (with bias) + RoPE + GQA
    attention (SDPA), SwiGLU MLP with fused gate+up, tied-free lm_head.
    Every projection is an nn.Linear, so F.linear hooks see all of them.
    ``model(ids, caches, pos)`` appends to KV caches from position ``pos``;
    a 0-d device tensor ``pos`` keeps every shape fixed (attention over the
    whole cache, later positions masked), so a decode step can be captured
    in a CUDA graph and replayed as ``pos`` advances.
    ``dtype``: bfloat16 (default) or float16, the reference driver's
    ``--dtype`` (qwen_abft_benchmark.py:26)."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    class RMSNorm(nn.Module):
        def __init__(self, h):
            super().__init__()
            self.weight = nn.Parameter(torch.ones(h))

        def forward(self, x):
            xf = x.float()
            return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg["eps"])).to(x.dtype) * self.weight

    def rope(x, cos, sin):  # x [T, H, D]
        x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
        return x * cos + torch.cat((-x2, x1), dim=-1) * sin

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            h, nh, nkv, hd, it = cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["inter"]
            self.ln1, self.ln2 = RMSNorm(h), RMSNorm(h)
            self.qkv = nn.Linear(h, (nh + 2 * nkv) * hd, bias=True)
            self.o = nn.Linear(nh * hd, h, bias=False)
            self.gate_up = nn.Linear(h, 2 * it, bias=False)
            self.down = nn.Linear(it, h, bias=False)

        def forward(self, x, cos, sin, cache=None, pos=0):
            nh, nkv, hd = cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
            t = x.shape[0]
            q, k, v = self.qkv(self.ln1(x)).split([nh * hd, nkv * hd, nkv * hd], dim=-1)
            q = rope(q.view(t, nh, hd), cos, sin).transpose(0, 1)
            k = rope(k.view(t, nkv, hd), cos, sin).transpose(0, 1)
            v = v.view(t, nkv, hd).transpose(0, 1)
            mask = None
            if cache is not None and torch.is_tensor(pos):
                # fixed shapes for a CUDA graph: pos lives on the device, and
                # attention runs over the whole cache with later positions masked
                at = pos + torch.arange(t, device=x.device)
                cache[0].index_copy_(1, at, k)
                cache[1].index_copy_(1, at, v)
                k, v = cache[0], cache[1]
                mask = torch.arange(cache.shape[2], device=x.device)[None, :] <= at[:, None]
            elif cache is not None:  # [2, nkv, T_max, hd]: keys and values of positions < pos + t
                cache[0, :, pos:pos + t] = k
                cache[1, :, pos:pos + t] = v
                k, v = cache[0, :, :pos + t], cache[1, :, :pos + t]
            a = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=(t > 1 and mask is None),
                                               enable_gqa=True)
            x = x + self.o(a.transpose(0, 1).reshape(t, nh * hd))
            g, u = self.gate_up(self.ln2(x)).chunk(2, dim=-1)
            return x + self.down(F.silu(g) * u)

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Embedding(cfg["vocab"], cfg["hidden"])
            self.layers = nn.ModuleList([Layer() for _ in range(cfg["layers"])])
            self.norm = RMSNorm(cfg["hidden"])
            self.lm_head = nn.Linear(cfg["hidden"], cfg["vocab"], bias=False)

        def forward(self, ids, caches=None, pos=0):
            t = ids.shape[0]
            hd = cfg["head_dim"]
            inv = 1.0 / (cfg["rope_theta"] ** (torch.arange(0, hd, 2, device=ids.device).float() / hd))
            at = pos + torch.arange(t, device=ids.device) if torch.is_tensor(pos) else \
                torch.arange(pos, pos + t, device=ids.device)
            ang = torch.outer(at.float(), inv)
            ang = torch.cat((ang, ang), dim=-1)[:, None, :]
            cos, sin = ang.cos().to(dt), ang.sin().to(dt)
            x = self.embed(ids)
            for i, layer in enumerate(self.layers):
                x = layer(x, cos, sin, None if caches is None else caches[i], pos)
            return self.lm_head(self.norm(x))

        def new_caches(self, t_max):
            return [torch.zeros(2, cfg["kv_heads"], t_max, cfg["head_dim"], dtype=dt,
                                device=self.embed.weight.device) for _ in range(cfg["layers"])]

    dt = torch.bfloat16 if dtype is None else dtype
    torch.manual_seed(seed)
    with torch.device(device):
        model = Model().to(dt)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, (nn.Linear, nn.Embedding)):
                mod.weight.normal_(0.0, 0.02)
                if getattr(mod, "bias", None) is not None:
                    mod.bias.zero_()
    return model.eval()



COGACT = dict(
    vit=dict(hidden=1024, mlp=4096, layers=24, heads=16),        # ViT-L/14 at 224^2
    siglip=dict(hidden=1152, mlp=4304, layers=27, heads=16),     # SigLIP-So400m/14 at 224^2
    llm=dict(hidden=4096, mlp=11008, layers=32, heads=32),       # Llama-2-7B
    dit=dict(hidden=768, mlp=3072, layers=12, heads=12),         # DiT-B action head
    patches=256, text_tokens=32, action_tokens=16, action_dim=7, denoise_steps=10, vocab=32000)


def build_cogact(cfg, device, seed=0):
    """Random-init CogACT-style VLA: two ViT encoders (patch conv, pre-norm
    blocks with fused QKV + GELU MLP), an MLP projector, a Llama-style
    decoder (RMSNorm, RoPE, fused QKV, SwiGLU with fused gate+up) and a
    DiT-B action head (adaLN-zero blocks conditioned on the decoder's last
    hidden state and the denoising step). Every projection is an nn.Linear."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    class RMSNorm(nn.Module):
        def __init__(self, h):
            super().__init__()
            self.weight = nn.Parameter(torch.ones(h))

        def forward(self, x):
            xf = x.float()
            return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype) * self.weight

    def attend(qkv, heads, causal, cos=None, sin=None):
        t, three_h = qkv.shape
        hd = three_h // 3 // heads
        q, k, v = qkv.view(t, 3, heads, hd).unbind(1)
        if cos is not None:
            def rope(x):
                x1, x2 = x[..., : hd // 2], x[..., hd // 2:]
                return x * cos + torch.cat((-x2, x1), dim=-1) * sin
            q, k = rope(q), rope(k)
        o = F.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1), is_causal=causal)
        return o.transpose(0, 1).reshape(t, heads * hd)

    class VitBlock(nn.Module):
        def __init__(self, c):
            super().__init__()
            h = c["hidden"]
            self.heads = c["heads"]
            self.n1, self.n2 = nn.LayerNorm(h), nn.LayerNorm(h)
            self.qkv, self.o = nn.Linear(h, 3 * h), nn.Linear(h, h)
            self.fc1, self.fc2 = nn.Linear(h, c["mlp"]), nn.Linear(c["mlp"], h)

        def forward(self, x):
            x = x + self.o(attend(self.qkv(self.n1(x)), self.heads, False))
            return x + self.fc2(F.gelu(self.fc1(self.n2(x)), approximate="tanh"))

    class Vit(nn.Module):
        def __init__(self, c):
            super().__init__()
            self.patch = nn.Conv2d(3, c["hidden"], kernel_size=14, stride=14)
            self.pos = nn.Parameter(torch.zeros(cfg["patches"], c["hidden"]))
            self.blocks = nn.ModuleList([VitBlock(c) for _ in range(c["layers"])])
            self.norm = nn.LayerNorm(c["hidden"])

        def forward(self, img):
            x = self.patch(img).flatten(2).transpose(1, 2)[0] + self.pos
            for b in self.blocks:
                x = b(x)
            return self.norm(x)

    class LlamaBlock(nn.Module):
        def __init__(self, c):
            super().__init__()
            h = c["hidden"]
            self.heads = c["heads"]
            self.n1, self.n2 = RMSNorm(h), RMSNorm(h)
            self.qkv, self.o = nn.Linear(h, 3 * h, bias=False), nn.Linear(h, h, bias=False)
            self.gate_up, self.down = nn.Linear(h, 2 * c["mlp"], bias=False), nn.Linear(c["mlp"], h, bias=False)

        def forward(self, x, cos, sin):
            x = x + self.o(attend(self.qkv(self.n1(x)), self.heads, True, cos, sin))
            g, u = self.gate_up(self.n2(x)).chunk(2, dim=-1)
            return x + self.down(F.silu(g) * u)

    class DitBlock(nn.Module):
        def __init__(self, c):
            super().__init__()
            h = c["hidden"]
            self.heads = c["heads"]
            self.n1 = nn.LayerNorm(h, elementwise_affine=False)
            self.n2 = nn.LayerNorm(h, elementwise_affine=False)
            self.qkv, self.o = nn.Linear(h, 3 * h), nn.Linear(h, h)
            self.fc1, self.fc2 = nn.Linear(h, c["mlp"]), nn.Linear(c["mlp"], h)
            self.ada = nn.Linear(h, 6 * h)

        def forward(self, x, c):
            s1, b1, g1, s2, b2, g2 = self.ada(F.silu(c)).chunk(6, dim=-1)
            x = x + g1 * self.o(attend(self.qkv(self.n1(x) * (1 + s1) + b1), self.heads, False))
            return x + g2 * self.fc2(F.gelu(self.fc1(self.n2(x) * (1 + s2) + b2), approximate="tanh"))

    class Vla(nn.Module):
        def __init__(self):
            super().__init__()
            v, s, l, d = cfg["vit"], cfg["siglip"], cfg["llm"], cfg["dit"]
            self.vit, self.siglip = Vit(v), Vit(s)
            self.proj1 = nn.Linear(v["hidden"] + s["hidden"], l["hidden"])
            self.proj2 = nn.Linear(l["hidden"], l["hidden"])
            self.embed = nn.Embedding(cfg["vocab"], l["hidden"])
            self.llm = nn.ModuleList([LlamaBlock(l) for _ in range(l["layers"])])
            self.llm_norm = RMSNorm(l["hidden"])
            self.cond = nn.Linear(l["hidden"], d["hidden"])
            self.t_embed = nn.Linear(256, d["hidden"])
            self.act_in = nn.Linear(cfg["action_dim"], d["hidden"])
            self.dit = nn.ModuleList([DitBlock(d) for _ in range(d["layers"])])
            self.act_out = nn.Linear(d["hidden"], cfg["action_dim"])

        def forward(self, img, text_ids, noise):
            vis = torch.cat((self.vit(img), self.siglip(img)), dim=-1)
            vis = self.proj2(F.gelu(self.proj1(vis), approximate="tanh"))
            x = torch.cat((vis, self.embed(text_ids)), dim=0)
            t, hd = x.shape[0], cfg["llm"]["hidden"] // cfg["llm"]["heads"]
            inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device=x.device).float() / hd))
            ang = torch.outer(torch.arange(t, device=x.device).float(), inv)
            ang = torch.cat((ang, ang), dim=-1)[:, None, :]
            cos, sin = ang.cos().to(x.dtype), ang.sin().to(x.dtype)
            for b in self.llm:
                x = b(x, cos, sin)
            cog = self.cond(self.llm_norm(x)[-1:])  # cognition feature of the last token
            a = noise
            for step in range(cfg["denoise_steps"]):
                freq = torch.exp(-torch.arange(128, device=x.device).float() * (9.21 / 128)) * (1000.0 * step)
                temb = torch.cat((freq.sin(), freq.cos()))[None].to(x.dtype)
                c = cog + self.t_embed(temb)
                h = self.act_in(a)
                for b in self.dit:
                    h = b(h, c)
                a = a - 0.1 * self.act_out(h)
            return a

    torch.manual_seed(seed)
    with torch.device(device):
        model = Vla().to(torch.bfloat16)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, (nn.Linear, nn.Embedding, nn.Conv2d)):
                mod.weight.normal_(0.0, 0.02)
                if getattr(mod, "bias", None) is not None:
                    mod.bias.zero_()
    return model.eval()
