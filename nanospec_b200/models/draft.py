"""DSPark draft: parameter schema, initialisation and the sharded weight tree.

The parameter names, shapes and the flat-shard element order are fixed by the
on-disk format shared with the reference (nanospec/dspark.py:20-68, 147-296):

* ``parameter_shapes`` lists every trainable tensor in TorchSpec naming order;
* ``initialize`` fills 1-D tensors with ones and the rest with N(0, 0.02) drawn
  from one CPU generator in that order (so both projects start from the same
  weights given the same seed);
* the trainable tensors form ``2 + num_hidden_layers`` *units*: ``context``
  (context_proj, context_norm, fc_norm.*), ``layers.i`` (layer-local names) and
  ``heads`` (final_norm, markov_head.*). Each unit is one flat buffer in the
  schema order, padded to ``ceil(n / N) * N`` elements, rank r owning
  ``[r*ss, (r+1)*ss)``.

The module tree (``context_proj``, ``layers[i].self_attn.q_proj`` ...) exists so
that parameters keep their public identities; while a unit is gathered its
parameters' ``.data`` are views into the gathered flat buffer.
"""

from __future__ import annotations

from collections import OrderedDict

import torch
from torch import nn

from ..config import DraftConfig
from ..parallel.shard import Shard, ShardingPlan

LAYER_KEYS = (
    "self_attn.q_proj.weight",
    "self_attn.k_proj.weight",
    "self_attn.v_proj.weight",
    "self_attn.o_proj.weight",
    "self_attn.q_norm.weight",
    "self_attn.k_norm.weight",
    "mlp.gate_proj.weight",
    "mlp.up_proj.weight",
    "mlp.down_proj.weight",
    "input_layernorm.weight",
    "post_attention_layernorm.weight",
)


def layer_shapes(c: DraftConfig) -> "OrderedDict[str, tuple]":
    h, d, m = c.hidden_size, c.head_dim, c.intermediate_size
    qd, kd = c.num_attention_heads * d, c.num_key_value_heads * d
    shapes = ((qd, h), (kd, h), (kd, h), (h, qd), (d,), (d,), (m, h), (m, h), (h, m), (h,), (h,))
    return OrderedDict(zip(LAYER_KEYS, shapes))


def parameter_shapes(c: DraftConfig) -> "OrderedDict[str, tuple]":
    """Every trainable tensor, in checkpoint order (nanospec/dspark.py:20-55)."""
    out = OrderedDict()
    out["context_proj.weight"] = (c.hidden_size, c.num_target_layers * c.target_hidden_size)
    out["context_norm.weight"] = (c.hidden_size,)
    if c.fc_norm:
        for i in range(c.num_target_layers):
            out[f"fc_norm.{i}.weight"] = (c.target_hidden_size,)
    per_layer = layer_shapes(c)
    for i in range(c.num_hidden_layers):
        for key, shape in per_layer.items():
            out[f"layers.{i}.{key}"] = shape
    out["final_norm.weight"] = (c.hidden_size,)
    if c.markov_rank:
        out["markov_head.markov_w1.weight"] = (c.vocab_size, c.markov_rank)
        out["markov_head.markov_w2.weight"] = (c.vocab_size, c.markov_rank)
    return out


@torch.no_grad()
def initialize(c: DraftConfig, seed: int = 42, dtype=torch.bfloat16) -> "OrderedDict[str, torch.Tensor]":
    """Reproducible initial weights: norms are ones, matrices N(0, 0.02) in schema order."""
    gen = torch.Generator().manual_seed(seed)
    state = OrderedDict()
    for name, shape in parameter_shapes(c).items():
        t = torch.empty(shape, dtype=dtype)
        if len(shape) == 1:
            t.fill_(1.0)
        else:
            t.normal_(0.0, 0.02, generator=gen)
        state[name] = t
    return state


class _Holder(nn.Module):
    """A named container whose single attribute ``weight`` is a registered Parameter.

    The parameter starts storage-less on the training device; its shard binds
    views of the gathered flat buffer into it.
    """

    def __init__(self, shape, f, eps=None):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(0, **f), requires_grad=False)
        self.shape = tuple(shape)
        if eps is not None:
            self.eps = eps


class DSparkAttention(nn.Module):
    def __init__(self, c: DraftConfig, f):
        super().__init__()
        s = layer_shapes(c)
        for key in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(self, key, _Holder(s[f"self_attn.{key}.weight"], f))
        self.q_norm = _Holder((c.head_dim,), f, c.rms_norm_eps)
        self.k_norm = _Holder((c.head_dim,), f, c.rms_norm_eps)


class DSparkMLP(nn.Module):
    def __init__(self, c: DraftConfig, f):
        super().__init__()
        s = layer_shapes(c)
        for key in ("gate_proj", "up_proj", "down_proj"):
            setattr(self, key, _Holder(s[f"mlp.{key}.weight"], f))


class DSparkDecoderLayer(nn.Module):
    def __init__(self, c: DraftConfig, f):
        super().__init__()
        self.self_attn = DSparkAttention(c, f)
        self.mlp = DSparkMLP(c, f)
        self.input_layernorm = _Holder((c.hidden_size,), f, c.rms_norm_eps)
        self.post_attention_layernorm = _Holder((c.hidden_size,), f, c.rms_norm_eps)


class MarkovHead(nn.Module):
    def __init__(self, vocab, rank, f):
        super().__init__()
        self.markov_w1 = _Holder((vocab, rank), f)
        self.markov_w2 = _Holder((vocab, rank), f)


class DSpark(nn.Module):
    """Trainable draft weights (sharded) plus the frozen target embedding and LM head.

    ``state`` holds the trainable tensors (``parameter_shapes`` keys); ``embedding``
    and ``lm_head`` are the frozen ``[vocab, hidden]`` target tensors, replicated on
    every training rank. ``group``/``world_size``/``rank`` describe the training
    process group the flat shards are split over.
    """

    def __init__(self, config: DraftConfig, state, embedding, lm_head, *, device,
                 dtype=torch.bfloat16, group=None, world_size=1, rank=0):
        super().__init__()
        c = self.config = config
        schema = parameter_shapes(c)
        if set(state) != set(schema) or any(tuple(state[k].shape) != schema[k] for k in schema):
            raise ValueError("Draft checkpoint keys/shapes do not match config")
        vh = (c.vocab_size, c.hidden_size)
        if tuple(embedding.shape) != vh or tuple(lm_head.shape) != vh:
            raise ValueError("Target embedding/head shape mismatch")
        self.dtype = dtype
        f = {"device": device, "dtype": dtype}
        self.context_proj = _Holder(schema["context_proj.weight"], f)
        self.context_norm = _Holder((c.hidden_size,), f, c.rms_norm_eps)
        self.fc_norm = nn.ModuleList(
            [_Holder((c.target_hidden_size,), f, c.rms_norm_eps) for _ in range(c.num_target_layers)]
            if c.fc_norm else []
        )
        self.layers = nn.ModuleList([DSparkDecoderLayer(c, f) for _ in range(c.num_hidden_layers)])
        self.final_norm = _Holder((c.hidden_size,), f, c.rms_norm_eps)
        self.markov_head = MarkovHead(c.vocab_size, c.markov_rank, f) if c.markov_rank else None
        self.requires_grad_(False)
        # Frozen, replicated target tensors.
        self.embed_tokens = _Holder(vh, f)
        self.embed_tokens.weight = nn.Parameter(
            embedding.detach().to(device=device, dtype=dtype).contiguous(), requires_grad=False)
        self.lm_head = _Holder(vh, f)
        self.lm_head.weight = nn.Parameter(
            lm_head.detach().to(device=device, dtype=dtype).contiguous(), requires_grad=False)

        place = dict(device=device, dtype=dtype, group=group, world_size=world_size, rank=rank)
        names = list(schema)
        ctx_names = [n for n in names if n.startswith(("context_", "fc_norm."))]
        head_names = [n for n in names if n.startswith(("final_norm.", "markov_head."))]
        entry = lambda mod, key, full: (key, mod.get_parameter(key), state[full])  # noqa: E731
        units = [Shard([entry(self, n, n) for n in ctx_names], shapes=schema, **place)]
        for i, layer in enumerate(self.layers):
            units.append(Shard([entry(layer, k, f"layers.{i}.{k}") for k in LAYER_KEYS],
                               shapes={k: schema[f"layers.{i}.{k}"] for k in LAYER_KEYS}, **place))
        units.append(Shard([entry(self, n, n) for n in head_names], shapes=schema, **place))
        self.sharding = ShardingPlan(units[0], tuple(units[1:-1]), units[-1])

    # ------------------------------------------------------------------ placement
    def _apply(self, fn, recurse=True):
        if not hasattr(self, "sharding"):
            return super()._apply(fn, recurse=recurse)
        # Parameters are views into the shards' flat buffers: move the owners, then rebind.
        if any(s.gathered is not None or s.full_grad is not None for s in self.sharding):
            raise RuntimeError("Release gathered buffers before moving the model")
        self.sharding.reset_pipeline()
        for s in self.sharding:
            s.apply_placement(fn)
        self.embed_tokens._apply(fn, recurse=recurse)
        self.lm_head._apply(fn, recurse=recurse)
        return self

    # ------------------------------------------------------------------ export
    @torch.no_grad()
    def draft_state_dict(self) -> "OrderedDict[str, torch.Tensor]":
        """TorchSpec-named trainable weights on CPU. Collective when sharded."""
        out = OrderedDict()
        for unit_name, shard in self.sharding.named_shards():
            prefix = unit_name + "." if unit_name.startswith("layers.") else ""
            for key, tensor in shard.gather().items():
                out[prefix + key] = tensor.detach().cpu().clone()
            shard.release()
        return out

    @torch.no_grad()
    def state_dict(self, *, destination=None, prefix="", keep_vars=False):
        """Full CPU state including the frozen embedding and LM head. Collective when sharded."""
        out = OrderedDict() if destination is None else destination
        for k, v in self.draft_state_dict().items():
            out[prefix + k] = v
        for name in ("embed_tokens.weight", "lm_head.weight"):
            p = self.get_parameter(name)
            out[prefix + name] = (p if keep_vars else p.detach()).cpu().clone()
        return out

    @torch.no_grad()
    def load_state_dict(self, state_dict, strict=True, assign=False):
        """Write each rank's slice of every tensor into its shard and reset the FP32 master."""
        if not hasattr(self, "sharding"):
            return super().load_state_dict(state_dict, strict=strict, assign=assign)
        if assign:
            raise ValueError("assign=True would replace parameters bound to manual shards")
        expected = dict(parameter_shapes(self.config))
        for name in ("embed_tokens.weight", "lm_head.weight"):
            expected[name] = tuple(self.get_parameter(name).shape)
        missing = sorted(set(expected) - set(state_dict))
        unexpected = sorted(set(state_dict) - set(expected))
        if strict and (missing or unexpected):
            raise RuntimeError(f"Missing keys: {missing}; unexpected keys: {unexpected}")
        for name in set(expected) & set(state_dict):
            if tuple(state_dict[name].shape) != tuple(expected[name]):
                raise RuntimeError(f"Shape mismatch for {name}: expected {expected[name]}")
        for unit_name, shard in self.sharding.named_shards():
            prefix = unit_name + "." if unit_name.startswith("layers.") else ""
            shard.load_tensors({k: state_dict[prefix + k] for k in shard.names if prefix + k in state_dict})
        for name in ("embed_tokens.weight", "lm_head.weight"):
            if name in state_dict:
                self.get_parameter(name).copy_(state_dict[name])
        return nn.modules.module._IncompatibleKeys(missing, unexpected)
