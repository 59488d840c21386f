"""Frozen Qwen3.5-style hybrid verifier: checkpoint I/O, weight containers, stage forward.

Checkpoint format: the Hugging Face layout the reference reads (nanospec/qwen.py:20-188):
``config.json`` (``model_type == "qwen3_5"``, ``text_config``, ``quantization_config``
with 128 x 128 ``weight_block_size`` and ``activation_scheme == "dynamic"``),
``model.safetensors.index.json`` and safetensors shards with names
``model.language_model.layers.{i}.(linear_attn|self_attn|mlp).*``,
``model.language_model.embed_tokens.weight``, ``model.language_model.norm.weight`` and
``lm_head.weight``. FP8 projections store ``weight`` (e4m3) and ``weight_scale_inv``
(fp32, one per 128 x 128 block).

``write_synthetic_checkpoint`` produces a random-init checkpoint of any shape in that
layout (there is no network for the real 27B weights); ``qwen3_5_27b_text_config``
gives the public 27B shapes used by the full-size benchmarks.

Execution (``stage_forward``) follows the reference's verifier loop
(nanospec/train.py:53-157): per layer, (1+w)-RMSNorm, then either the gated DeltaNet
branch (FP8 in-projections, causal depthwise conv + SiLU, L2-normalised q/k, chunked
gated delta rule, gated RMSNorm, FP8 out-projection) or full attention (q/gate
projection, per-head (1+w)-norm, partial RoPE, causal GQA, sigmoid gate, FP8
o-projection), residual, (1+w)-RMSNorm and the FP8 SwiGLU MLP.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch
from torch import nn

from .. import ops as _ops  # noqa: F401  (ensures the op package is importable)
from ..ops import verifier_ops as vops

PREFIX = "model.language_model."


# ---------------------------------------------------------------------------- configs
def qwen3_5_27b_text_config() -> dict:
    """Public Qwen3.5-27B text shapes: 64 layers, 3:1 GDN:attention, hidden 5120."""
    layers = 64
    return {
        "hidden_size": 5120,
        "intermediate_size": 17408,
        "num_hidden_layers": layers,
        "vocab_size": 248320,
        "rms_norm_eps": 1e-6,
        "layer_types": ["full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(layers)],
        "head_dim": 256,
        "num_attention_heads": 24,
        "num_key_value_heads": 4,
        "rope_parameters": {"rope_type": "default", "rope_theta": 10000000.0, "partial_rotary_factor": 0.25},
        "linear_num_key_heads": 16,
        "linear_num_value_heads": 48,
        "linear_key_head_dim": 128,
        "linear_value_head_dim": 128,
        "linear_conv_kernel_dim": 4,
    }


def tiny_hybrid_text_config(hidden=64, vocab=512, heads=4, head_dim=16, ffn=128) -> dict:
    """Four layers [GDN, GDN, GDN, attention] at a test-sized width."""
    return {
        "hidden_size": hidden,
        "intermediate_size": ffn,
        "num_hidden_layers": 4,
        "vocab_size": vocab,
        "rms_norm_eps": 1e-6,
        "layer_types": ["linear_attention"] * 3 + ["full_attention"],
        "head_dim": head_dim,
        "num_attention_heads": heads,
        "num_key_value_heads": max(1, heads // 2),
        "rope_parameters": {"rope_type": "default", "rope_theta": 1000000.0, "partial_rotary_factor": 0.5},
        "linear_num_key_heads": max(1, heads // 2),
        "linear_num_value_heads": heads,
        "linear_key_head_dim": head_dim,
        "linear_value_head_dim": head_dim,
        "linear_conv_kernel_dim": 4,
    }


def layer_tensor_shapes(tc: dict, i: int) -> dict:
    """Name -> (shape, fp8?) for decoder layer i (names without the model prefix)."""
    h, m = tc["hidden_size"], tc["intermediate_size"]
    p = f"layers.{i}."
    out = {p + "input_layernorm.weight": ((h,), False), p + "post_attention_layernorm.weight": ((h,), False)}
    if tc["layer_types"][i] == "linear_attention":
        nk, nv = tc["linear_num_key_heads"], tc["linear_num_value_heads"]
        dk, dv = tc["linear_key_head_dim"], tc["linear_value_head_dim"]
        conv = 2 * nk * dk + nv * dv
        a = p + "linear_attn."
        out.update({
            a + "in_proj_qkv": ((conv, h), True),
            a + "in_proj_z": ((nv * dv, h), True),
            a + "in_proj_b": ((nv, h), False),
            a + "in_proj_a": ((nv, h), False),
            a + "out_proj": ((h, nv * dv), True),
            a + "conv1d.weight": ((conv, 1, tc["linear_conv_kernel_dim"]), False),
            a + "A_log": ((nv,), False),
            a + "dt_bias": ((nv,), False),
            a + "norm.weight": ((dv,), False),
        })
    else:
        d, hq, hk = tc["head_dim"], tc["num_attention_heads"], tc["num_key_value_heads"]
        a = p + "self_attn."
        out.update({
            a + "q_proj": ((2 * hq * d, h), True),
            a + "k_proj": ((hk * d, h), True),
            a + "v_proj": ((hk * d, h), True),
            a + "o_proj": ((h, hq * d), True),
            a + "q_norm.weight": ((d,), False),
            a + "k_norm.weight": ((d,), False),
        })
    for name, shape in (("gate_proj", (m, h)), ("up_proj", (m, h)), ("down_proj", (h, m))):
        out[p + "mlp." + name] = (shape, True)
    return out


# ---------------------------------------------------------------------------- checkpoint
class Checkpoint:
    """Reads an HF-layout checkpoint directory (config + safetensors index)."""

    def __init__(self, path):
        self.path = Path(path)
        self.config = json.loads((self.path / "config.json").read_text())
        self.index = json.loads((self.path / "model.safetensors.index.json").read_text())["weight_map"]

    @property
    def text_config(self) -> dict:
        return self.config["text_config"]

    def load(self, keys, device="cpu") -> dict:
        from safetensors import safe_open
        by_file = {}
        for key in keys:
            by_file.setdefault(self.index[key], []).append(key)
        out = {}
        for fname, names in by_file.items():
            with safe_open(str(self.path / fname), framework="pt", device="cpu") as f:
                for name in names:
                    out[name] = f.get_tensor(name).to(device)
        return out

    def frozen(self, device="cpu") -> dict:
        return self.load([PREFIX + "embed_tokens.weight", "lm_head.weight"], device)


def quantize_weight_blocks(w: torch.Tensor, block=128):
    """fp32 weight -> (e4m3 weight, fp32 weight_scale_inv per 128 x 128 block)."""
    n, k = w.shape
    wb = w.float().view(n // block, block, k // block, block)
    s = wb.abs().amax(dim=(1, 3)) / 448.0
    s = torch.where(s > 0, s, torch.ones_like(s))
    q = (wb / s[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q.view(n, k), s.float()


@torch.no_grad()
def write_synthetic_checkpoint(path, text_config: dict, *, seed=0, fp8=True, std=0.02,
                               shard_bytes=4 << 30, dtype=torch.bfloat16, device="cpu") -> Path:
    """Random-init checkpoint in the HF Qwen3.5 FP8 layout.

    ``fp8=False`` keeps projections in ``dtype`` (needed when widths are not multiples
    of 128). Norm weights are small random offsets (the (1+w) convention), A_log and
    dt_bias follow the usual GDN initialisation ranges. ``device="cuda"`` draws and
    quantizes the tensors on the GPU (a 27B-shaped checkpoint takes seconds instead
    of many minutes); the files are the same format either way.
    """
    from safetensors.torch import save_file
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    tc = dict(text_config)
    gen = torch.Generator(device=device).manual_seed(seed)
    h, v = tc["hidden_size"], tc["vocab_size"]
    shard, shard_size, files, weight_map = {}, 0, [], {}
    rand = lambda shape: torch.randn(shape, generator=gen, device=device)  # noqa: E731

    def flush():
        nonlocal shard, shard_size
        if not shard:
            return
        name = f"model-{len(files) + 1:05d}.safetensors"
        save_file(shard, str(path / name))
        for k in shard:
            weight_map[k] = name
        files.append(name)
        shard, shard_size = {}, 0

    def put(name, t):
        nonlocal shard_size
        shard[name] = t.contiguous().cpu()
        shard_size += t.numel() * t.element_size()
        if shard_size >= shard_bytes:
            flush()

    put(PREFIX + "embed_tokens.weight", (rand((v, h)) * std).to(dtype))
    for i in range(tc["num_hidden_layers"]):
        for name, (shape, quant) in layer_tensor_shapes(tc, i).items():
            full = PREFIX + name
            if name.endswith("A_log"):
                put(full, torch.log(torch.empty(shape, device=device).uniform_(1, 16, generator=gen)).float())
            elif name.endswith("dt_bias"):
                put(full, (torch.rand(shape, generator=gen, device=device) * 0.5).float())
            elif name.endswith("conv1d.weight"):
                put(full, (rand(shape) * 0.3).to(dtype))
            elif len(shape) == 1:
                put(full, (rand(shape) * 0.05).to(dtype))
            else:
                w = rand(shape) * std
                if quant and fp8 and shape[0] % 128 == 0 and shape[1] % 128 == 0:
                    q, s = quantize_weight_blocks(w)
                    put(full + ".weight", q)
                    put(full + ".weight_scale_inv", s)
                else:
                    put(full + ".weight", w.to(dtype))
                del w
    put(PREFIX + "norm.weight", (rand(h) * 0.05).to(dtype))
    put("lm_head.weight", (rand((v, h)) * std).to(dtype))
    flush()
    config = synthetic_hf_config(tc, seed=seed, fp8=fp8)
    (path / "config.json").write_text(json.dumps(config, indent=2))
    (path / "model.safetensors.index.json").write_text(
        json.dumps({"metadata": {}, "weight_map": weight_map}, indent=2))
    return path


# ---------------------------------------------------------------------------- containers
class _W(nn.Module):
    def __init__(self, weight, eps=None):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        if eps is not None:
            self.eps = eps


class FP8Linear(nn.Module):
    """Projection with an e4m3 weight and a per-block ``weight_scale_inv`` (or a plain weight)."""

    def __init__(self, weight, scale=None):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.register_buffer("weight_scale_inv", scale)

    @classmethod
    def load(cls, w, prefix):
        return cls(w[prefix + ".weight"], w.get(prefix + ".weight_scale_inv"))


class QwenGatedDeltaNet(nn.Module):
    def __init__(self, tc, w, p):
        super().__init__()
        self.num_key_heads = tc["linear_num_key_heads"]
        self.num_value_heads = tc["linear_num_value_heads"]
        self.key_head_dim = tc["linear_key_head_dim"]
        self.value_head_dim = tc["linear_value_head_dim"]
        for name in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
            setattr(self, name, FP8Linear.load(w, p + name))
        self.conv1d = _W(w[p + "conv1d.weight"])
        self.A_log = nn.Parameter(w[p + "A_log"], requires_grad=False)
        self.dt_bias = nn.Parameter(w[p + "dt_bias"], requires_grad=False)
        self.norm = _W(w[p + "norm.weight"], tc["rms_norm_eps"])


class QwenAttention(nn.Module):
    def __init__(self, tc, w, p):
        super().__init__()
        self.head_dim = tc["head_dim"]
        self.num_heads = tc["num_attention_heads"]
        self.num_key_value_heads = tc["num_key_value_heads"]
        rope = tc["rope_parameters"]
        self.rotary_dim = int(self.head_dim * rope.get("partial_rotary_factor", 1.0))
        self.rope_theta = rope["rope_theta"]
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(self, name, FP8Linear.load(w, p + name))
        self.q_norm = _W(w[p + "q_norm.weight"], tc["rms_norm_eps"])
        self.k_norm = _W(w[p + "k_norm.weight"], tc["rms_norm_eps"])


class QwenMLP(nn.Module):
    def __init__(self, w, p):
        super().__init__()
        for name in ("gate_proj", "up_proj", "down_proj"):
            setattr(self, name, FP8Linear.load(w, p + name))


class QwenDecoderLayer(nn.Module):
    def __init__(self, tc, w, i):
        super().__init__()
        p = f"layers.{i}."
        eps = tc["rms_norm_eps"]
        self.input_layernorm = _W(w[p + "input_layernorm.weight"], eps)
        self.post_attention_layernorm = _W(w[p + "post_attention_layernorm.weight"], eps)
        if tc["layer_types"][i] == "linear_attention":
            self.linear_attn, self.self_attn = QwenGatedDeltaNet(tc, w, p + "linear_attn."), None
        else:
            self.linear_attn, self.self_attn = None, QwenAttention(tc, w, p + "self_attn.")
        self.mlp = QwenMLP(w, p + "mlp.")


class QwenStage(nn.Module):
    """Contiguous layer range [start, end) of the verifier, with embed (first) / norm+head (last).

    Weights come from ``checkpoint`` (HF layout, as the reference's ``QwenStage``,
    nanospec/qwen.py:144-188) or, with ``checkpoint=None``, from ``weights`` (names
    without the ``model.language_model.`` prefix) and ``config`` (a full HF
    ``config.json`` dict), e.g. ``random_verifier_weights``.
    """

    def __init__(self, checkpoint: Checkpoint | None, start, end, *, device, first=False, last=False,
                 weights: dict | None = None, config: dict | None = None):
        super().__init__()
        cfg = checkpoint.config if checkpoint is not None else config
        tc = self.config = cfg["text_config"]
        if cfg.get("model_type") != "qwen3_5":
            raise ValueError("Only the dense Qwen3.5 text backbone is implemented")
        quant = cfg.get("quantization_config", {})
        if quant.get("weight_block_size") != [128, 128] or quant.get("activation_scheme") != "dynamic":
            raise ValueError("Expected a dynamic 128x128 block-FP8 Qwen checkpoint")
        if tc["rope_parameters"].get("rope_type", "default") != "default":
            raise ValueError("Only default RoPE is supported")
        self.start, self.end = start, end
        if checkpoint is not None:
            keys = [k for k in checkpoint.index
                    if any(k.startswith(f"{PREFIX}layers.{i}.") for i in range(start, end))]
            if first:
                keys.append(PREFIX + "embed_tokens.weight")
            if last:
                keys += [PREFIX + "norm.weight", "lm_head.weight"]
            loaded = checkpoint.load(keys, device)
            w = {(k[len(PREFIX):] if k.startswith(PREFIX) else k): v for k, v in loaded.items()}
        else:
            w = weights
        self.layers = nn.ModuleList([QwenDecoderLayer(tc, w, i) for i in range(start, end)])
        self.embed_tokens = _W(w["embed_tokens.weight"]) if first else None
        self.norm = _W(w["norm.weight"], tc["rms_norm_eps"]) if last else None
        self.lm_head = _W(w["lm_head.weight"]) if last else None
        self.eval()
        self.fused = False
        if torch.device(device).type == "cuda":
            fuse_projections(self)
            self.fused = _fused_ok(self)


def _is_fp8(lin) -> bool:
    w = lin.weight
    return w.dtype == torch.float8_e4m3fn and w.shape[0] % 128 == 0 and w.shape[1] % 128 == 0


@torch.no_grad()
def _fuse(parts):
    """One projection over adjacent weights (same input): the parts become row views of
    the fused weight and scale, so the memory is not duplicated."""
    w = torch.cat([p.weight for p in parts], 0)
    fp8 = parts[0].weight_scale_inv is not None
    sc = torch.cat([p.weight_scale_inv for p in parts], 0) if fp8 else None
    r = 0
    for p in parts:
        n = p.weight.shape[0]
        p.weight = nn.Parameter(w[r:r + n], requires_grad=False)
        if fp8:
            p.weight_scale_inv = sc[r // 128:(r + n) // 128]
        r += n
    return FP8Linear(w, sc)


def fuse_projections(stage: "QwenStage"):
    """Concatenate projections that read the same input (once, on CUDA stages):
    GDN [in_proj_qkv; in_proj_z] and [in_proj_b; in_proj_a], attention [q; k; v], MLP
    [gate; up]. The fused forward runs one GEMM for each group."""
    for layer in stage.layers:
        a = layer.linear_attn
        if a is not None and _is_fp8(a.in_proj_qkv) and _is_fp8(a.in_proj_z):
            a.in_proj_qkvz = _fuse([a.in_proj_qkv, a.in_proj_z])
            a.in_proj_ba = _fuse([a.in_proj_b, a.in_proj_a])
        t = layer.self_attn
        if t is not None and all(_is_fp8(p) for p in (t.q_proj, t.k_proj, t.v_proj)):
            t.qkv = _fuse([t.q_proj, t.k_proj, t.v_proj])
        m = layer.mlp
        if _is_fp8(m.gate_proj) and _is_fp8(m.up_proj) and _is_fp8(m.down_proj):
            m.gate_up = _fuse([m.gate_proj, m.up_proj])


def _fused_ok(stage) -> bool:
    return all(getattr(l.mlp, "gate_up", None) is not None and
               (getattr(l.linear_attn, "in_proj_qkvz", None) is not None if l.linear_attn is not None
                else getattr(l.self_attn, "qkv", None) is not None)
               for l in stage.layers) and stage.config["hidden_size"] % 128 == 0 and \
        stage.config.get("linear_value_head_dim", 128) == 128


def synthetic_hf_config(text_config: dict, *, seed=0, fp8=True) -> dict:
    """The ``config.json`` dict of a synthetic Qwen3.5 FP8 checkpoint."""
    return {
        "model_type": "qwen3_5",
        "architectures": ["Qwen3_5ForConditionalGeneration"],
        "text_config": dict(text_config),
        "quantization_config": {"quant_method": "fp8", "weight_block_size": [128, 128],
                                "activation_scheme": "dynamic", "fmt": "e4m3"},
        "synthetic": {"seed": seed, "fp8": fp8},
    }


@torch.no_grad()
def random_verifier_weights(text_config: dict, start: int, end: int, *, device, first=False, last=False,
                            seed=0, std=0.02, dtype=torch.bfloat16, embed=None, lm_head=None) -> dict:
    """Random-init weights of layers [start, end) generated on ``device`` (no checkpoint).

    Same value ranges as ``write_synthetic_checkpoint``; FP8 projections are
    quantized per 128 x 128 block on the device. ``embed`` / ``lm_head``, when
    given, are used instead of fresh tensors (so a draft and the verifier can share
    the frozen target tensors).
    """
    tc = text_config
    gen = torch.Generator(device=device).manual_seed(seed)
    h, v = tc["hidden_size"], tc["vocab_size"]
    out = {}
    for i in range(start, end):
        for name, (shape, quant) in layer_tensor_shapes(tc, i).items():
            if name.endswith("A_log"):
                out[name] = torch.log(torch.empty(shape, device=device).uniform_(1, 16, generator=gen))
            elif name.endswith("dt_bias"):
                out[name] = torch.rand(shape, device=device, generator=gen) * 0.5
            elif name.endswith("conv1d.weight"):
                out[name] = (torch.randn(shape, device=device, generator=gen) * 0.3).to(dtype)
            elif len(shape) == 1:
                out[name] = (torch.randn(shape, device=device, generator=gen) * 0.05).to(dtype)
            else:
                w = torch.randn(shape, device=device, generator=gen) * std
                if quant and shape[0] % 128 == 0 and shape[1] % 128 == 0:
                    q, sc = quantize_weight_blocks(w)
                    out[name + ".weight"], out[name + ".weight_scale_inv"] = q, sc
                else:
                    out[name + ".weight"] = w.to(dtype)
                del w
    if first:
        out["embed_tokens.weight"] = embed if embed is not None else \
            (torch.randn(v, h, device=device, generator=gen) * std).to(dtype)
    if last:
        out["norm.weight"] = (torch.randn(h, device=device, generator=gen) * 0.05).to(dtype)
        out["lm_head.weight"] = lm_head if lm_head is not None else \
            (torch.randn(v, h, device=device, generator=gen) * std).to(dtype)
    return out


# ---------------------------------------------------------------------------- execution
@torch.no_grad()
def gdn_forward(attn: QwenGatedDeltaNet, n):
    b, s, _ = n.shape
    nk, nv = attn.num_key_heads, attn.num_value_heads
    dk, dv = attn.key_head_dim, attn.value_head_dim
    mixed = vops.fp8_linear(n, attn.in_proj_qkv.weight, attn.in_proj_qkv.weight_scale_inv)
    z = vops.fp8_linear(n, attn.in_proj_z.weight, attn.in_proj_z.weight_scale_inv)
    bpre = vops.fp8_linear(n, attn.in_proj_b.weight, attn.in_proj_b.weight_scale_inv)
    apre = vops.fp8_linear(n, attn.in_proj_a.weight, attn.in_proj_a.weight_scale_inv)
    mixed = vops.causal_conv_silu(mixed, attn.conv1d.weight)
    q, k, v = mixed.split((nk * dk, nk * dk, nv * dv), -1)
    q = q.reshape(b, s, nk, dk)
    k = k.reshape(b, s, nk, dk)
    v = v.reshape(b, s, nv, dv)
    g, beta = vops.gdn_gates(apre, bpre, attn.A_log, attn.dt_bias)
    out = vops.gated_delta_rule(q, k, v, g, beta, nv // nk)
    out = vops.qwen_gated_norm(out.reshape(-1, dv), z.reshape(-1, dv), attn.norm.weight, attn.norm.eps)
    return vops.fp8_linear(out.reshape(b, s, nv * dv), attn.out_proj.weight, attn.out_proj.weight_scale_inv)


@torch.no_grad()
def attention_forward(attn: QwenAttention, n):
    b, s, _ = n.shape
    d, hq, hk = attn.head_dim, attn.num_heads, attn.num_key_value_heads
    qg = vops.fp8_linear(n, attn.q_proj.weight, attn.q_proj.weight_scale_inv).view(b, s, hq, 2 * d)
    k = vops.fp8_linear(n, attn.k_proj.weight, attn.k_proj.weight_scale_inv).view(b, s, hk, d)
    v = vops.fp8_linear(n, attn.v_proj.weight, attn.v_proj.weight_scale_inv).view(b, s, hk, d)
    pos = torch.arange(s, device=n.device).expand(b, s)
    cos, sin = vops.rotary_factors(pos, attn.rotary_dim, attn.rope_theta, n.dtype)
    out = vops.gated_attention(qg, k, v, attn.q_norm.weight, attn.k_norm.weight, attn.q_norm.eps, cos, sin,
                               attn.rotary_dim)
    return vops.fp8_linear(out.reshape(b, s, hq * d), attn.o_proj.weight, attn.o_proj.weight_scale_inv)


@torch.no_grad()
def _gdn_fused(attn: QwenGatedDeltaNet, n_bf, nq, b, s):
    nk, nv = attn.num_key_heads, attn.num_value_heads
    dk, dv = attn.key_head_dim, attn.value_head_dim
    conv = 2 * nk * dk + nv * dv
    mixed = vops.fp8_gemm(nq[0], nq[1], attn.in_proj_qkvz.weight, attn.in_proj_qkvz.weight_scale_inv)
    ba = vops.fp8_linear(n_bf, attn.in_proj_ba.weight, None)
    total = mixed.shape[1]
    qkv = vops.causal_conv_silu_rows(mixed.view(b, s, total), total, attn.conv1d.weight, conv)
    q, k, v = qkv.split((nk * dk, nk * dk, nv * dv), -1)
    g, beta = vops.gdn_gates(ba[:, nv:].contiguous(), ba[:, :nv].contiguous(), attn.A_log, attn.dt_bias)
    o = vops.gated_delta_rule(q.reshape(b, s, nk, dk), k.reshape(b, s, nk, dk), v.reshape(b, s, nv, dv),
                              g.view(b, s, nv), beta.view(b, s, nv), nv // nk)
    oq = vops.gated_norm_quantize(o.view(-1, dv), mixed[:, conv:], nv, total, attn.norm.weight, attn.norm.eps)
    return vops.fp8_gemm(oq[0].view(b * s, nv * dv), oq[1].view(b * s, nv), attn.out_proj.weight,
                         attn.out_proj.weight_scale_inv)


@torch.no_grad()
def _attention_fused(attn: QwenAttention, nq, b, s, device, dtype):
    d, hq, hk = attn.head_dim, attn.num_heads, attn.num_key_value_heads
    qkv = vops.fp8_gemm(nq[0], nq[1], attn.qkv.weight, attn.qkv.weight_scale_inv)
    total = qkv.shape[1]
    qkv3 = qkv.view(b, s, total)
    qg = qkv3[..., :2 * hq * d].unflatten(-1, (hq, 2 * d))
    k = qkv3[..., 2 * hq * d:2 * hq * d + hk * d].unflatten(-1, (hk, d))
    v = qkv3[..., 2 * hq * d + hk * d:].unflatten(-1, (hk, d))
    pos = torch.arange(s, device=device).expand(b, s)
    cos, sin = vops.rotary_factors(pos, attn.rotary_dim, attn.rope_theta, dtype)
    out = vops.gated_attention(qg, k, v, attn.q_norm.weight, attn.k_norm.weight, attn.q_norm.eps, cos, sin,
                               attn.rotary_dim)
    oq = vops.quantize(out.view(b * s, hq * d))
    return vops.fp8_gemm(oq[0], oq[1], attn.o_proj.weight, attn.o_proj.weight_scale_inv)


@torch.no_grad()
def _stage_forward_fused(stage: QwenStage, x, capture, on_capture, handoff=None):
    """CUDA forward with fused projections and fused producers: every residual add is
    fused with the following (1+w)-RMSNorm, and every FP8 projection input leaves its
    producer already quantised (e4m3 + 1 x 128 scales). Same math as the statement
    path below; only roundings inside fp32 reductions differ.

    ``handoff``: ``{layer index or "final": (window id, rank, byte offset)}``; the
    add+norm kernel that produces a captured residual (or the final normed hidden
    state) also stores it into that rank's peer window, and the entry is removed
    (entries left over were produced by other kernels: the caller copies them)."""
    b, s, h = x.shape
    handoff = {} if handoff is None else handoff

    def peer(li, final):
        xt = handoff.pop(li) if li in capture and li in handoff else None
        nt = handoff.pop("final") if final and "final" in handoff else None
        if xt is None and nt is None:
            return None
        win = (xt or nt)[0]
        return (win, None if xt is None else xt[1:], None if nt is None else nt[1:])
    layers = list(stage.layers)
    ln = layers[0].input_layernorm
    _, n_bf, nq = vops.add_norm(x, None, ln.weight, ln.eps, want_bf16=layers[0].linear_attn is not None,
                                want_q=True)
    captured = {}
    for i, layer in enumerate(layers):
        li = stage.start + i
        if layer.linear_attn is not None:
            out = _gdn_fused(layer.linear_attn, n_bf.view(b * s, h), (nq[0], nq[1]), b, s)
        else:
            out = _attention_fused(layer.self_attn, nq, b, s, x.device, x.dtype)
        pl = layer.post_attention_layernorm
        x, _, n2q = vops.add_norm(x, out.view(b, s, h), pl.weight, pl.eps, want_bf16=False, want_q=True)
        mlp = layer.mlp
        gu = vops.fp8_gemm(n2q[0], n2q[1], mlp.gate_up.weight, mlp.gate_up.weight_scale_inv)
        hq = vops.silu_mul_quantize(gu)
        down = vops.fp8_gemm(hq[0], hq[1], mlp.down_proj.weight, mlp.down_proj.weight_scale_inv).view(b, s, h)
        if i + 1 < len(layers):
            nxt = layers[i + 1]
            ln = nxt.input_layernorm
            x, n_bf, nq = vops.add_norm(x, down, ln.weight, ln.eps, want_bf16=nxt.linear_attn is not None,
                                        want_q=True, peer=peer(li, False))
        elif stage.norm is not None:
            x, final, _ = vops.add_norm(x, down, stage.norm.weight, stage.norm.eps, peer=peer(li, True))
        else:
            x = vops.add(x, down)
        if li in capture:
            captured[li] = x
            if on_capture is not None:
                on_capture(li, x)
    return (final if stage.norm is not None else x), captured


@torch.no_grad()
def stage_forward(stage: QwenStage, x_or_ids, capture=(), on_capture=None, handoff=None):
    """Run the stage's layers. Returns (output, {layer_index: hidden}).

    ``x_or_ids``: token ids [b, s] for the first stage, else the hidden state [b, s, H].
    ``on_capture(layer_index, hidden)``, when given, receives each captured decoder
    output as soon as it exists (used to start the trainer hand-off early).
    ``handoff`` (fused CUDA path): see ``_stage_forward_fused``.
    """
    if stage.embed_tokens is not None:
        x = vops.embedding(x_or_ids, stage.embed_tokens.weight)
    else:
        x = x_or_ids
    if getattr(stage, "fused", False) and x.is_cuda and len(stage.layers) > 0:
        return _stage_forward_fused(stage, x, capture, on_capture, handoff)
    captured = {}
    for li, layer in enumerate(stage.layers, start=stage.start):
        n = vops.qwen_norm(x, layer.input_layernorm.weight, layer.input_layernorm.eps)
        out = gdn_forward(layer.linear_attn, n) if layer.linear_attn is not None else attention_forward(layer.self_attn, n)
        x = vops.add(x, out)
        n = vops.qwen_norm(x, layer.post_attention_layernorm.weight, layer.post_attention_layernorm.eps)
        mlp = layer.mlp
        gate = vops.fp8_linear(n, mlp.gate_proj.weight, mlp.gate_proj.weight_scale_inv)
        up = vops.fp8_linear(n, mlp.up_proj.weight, mlp.up_proj.weight_scale_inv)
        x = vops.add(x, vops.fp8_linear(vops.silu_mul(gate, up), mlp.down_proj.weight, mlp.down_proj.weight_scale_inv))
        if li in capture:
            captured[li] = x
            if on_capture is not None:
                on_capture(li, x)
    if stage.norm is not None:
        x = vops.qwen_norm(x, stage.norm.weight, stage.norm.eps)
    return x, captured


def verifier_flops_per_token(tc: dict, seq: int) -> float:
    """Rough forward FLOPs per token (projections + attention/GDN mixing), for roofline notes."""
    h, m = tc["hidden_size"], tc["intermediate_size"]
    total = 0.0
    for t in tc["layer_types"]:
        total += 2 * 3 * h * m
        if t == "linear_attention":
            nk, nv = tc["linear_num_key_heads"], tc["linear_num_value_heads"]
            dk, dv = tc["linear_key_head_dim"], tc["linear_value_head_dim"]
            total += 2 * h * (2 * nk * dk + 2 * nv * dv + 2 * nv) + 2 * nv * dv * h
            total += 2 * nv * (4 * dk * dv + 2 * 64 * (dk + dv))
        else:
            d, hq, hk = tc["head_dim"], tc["num_attention_heads"], tc["num_key_value_heads"]
            total += 2 * h * (2 * hq * d + 2 * hk * d) + 2 * hq * d * h + 2 * hq * d * seq
    return total
