"""Draft, objective and GPU-layout configuration.

Field names and validation rules are those of the reference's dataclasses
(nanospec/config.py:9-66) so JSON configs interchange between the two projects;
the checkpoint metadata stores ``DraftConfig.to_dict()`` verbatim.
``Topology`` is new: it describes how the GPUs of one box are split between
verifier partitions and training ranks (the reference hard-wires 8 ranks,
nanospec/distributed.py:15-28).
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from pathlib import Path

# Revision pins recorded in checkpoint metadata (nanospec/config.py:5-7). They name
# the upstream artefacts whose layout this runtime reproduces; nothing is downloaded.
TORCHSPEC_REVISION = "076a738fdd7e64be1495338f055e8188784633c4"
TARGET_MODEL = "Qwen/Qwen3.5-27B-FP8"
TARGET_REVISION = "709d2d2a46f204254221f583f45e00f93b578c9e"

CONFIG_DIR = Path(__file__).resolve().parent / "configs"


@dataclass
class DraftConfig:
    """DSPark draft shape. Defaults are the 5-layer 1.75 B-parameter Qwen draft."""

    hidden_size: int = 5120
    intermediate_size: int = 15360
    num_hidden_layers: int = 5
    num_attention_heads: int = 40
    num_key_value_heads: int = 8
    head_dim: int = 128
    vocab_size: int = 248320
    target_hidden_size: int = 5120
    target_num_hidden_layers: int = 64
    num_target_layers: int = 5
    target_layer_ids: tuple[int, ...] = (1, 16, 31, 46, 61)
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000000.0
    max_position_embeddings: int = 262144
    mask_token_id: int = 248063
    markov_rank: int = 256
    markov_head_type: str = "vanilla"
    fc_norm: bool = False
    tie_word_embeddings: bool = False

    def __post_init__(self):
        self.target_layer_ids = tuple(int(i) for i in self.target_layer_ids)
        problems = []
        if self.hidden_size != self.target_hidden_size:
            problems.append("the frozen target embedding/LM head need draft width == target width")
        if self.num_attention_heads % self.num_key_value_heads:
            problems.append("query heads must be a multiple of key/value heads")
        if self.head_dim % 2:
            problems.append("rotary embedding needs an even head_dim")
        if len(self.target_layer_ids) != self.num_target_layers:
            problems.append("target_layer_ids length must equal num_target_layers")
        if any(not 0 <= i < self.target_num_hidden_layers for i in self.target_layer_ids):
            problems.append("target_layer_ids index decoder outputs, zero based, in range")
        if self.markov_head_type != "vanilla" or self.markov_rank < 0:
            problems.append("only the vanilla Markov head (rank >= 0) exists")
        if not 0 <= self.mask_token_id < self.vocab_size:
            problems.append("mask_token_id must lie inside the vocabulary")
        if problems:
            raise ValueError("; ".join(problems))

    @classmethod
    def load(cls, path) -> "DraftConfig":
        with open(path) as f:
            return cls(**json.load(f))

    def to_dict(self) -> dict:
        d = asdict(self)
        d["target_layer_ids"] = list(self.target_layer_ids)
        return d


@dataclass
class Objective:
    """0.1 CE + 0.9 KL(target || draft) with exp(-slot/gamma) slot weights."""

    block_size: int = 7
    num_anchors: int = 32
    gamma: float = 4.0
    ce: float = 0.1
    kl: float = 0.9

    def __post_init__(self):
        if self.block_size < 1 or self.num_anchors < 1:
            raise ValueError("block_size and num_anchors must be positive")
        if self.ce < 0 or self.kl < 0:
            raise ValueError("loss weights must be non-negative")


@dataclass
class Topology:
    """Split of one box's GPUs into verifier partitions and training ranks.

    ``train_gpus`` training ranks take global ranks ``0..N-1``; the remaining
    ``world - N`` ranks own contiguous verifier layer ranges, in order. With
    ``colocate=True`` (1-GPU boxes, or when every GPU trains) the verifier runs
    on the training ranks themselves, partitioned over them.

    ``replicate=True`` is the layout a 180 GB GPU makes possible: every training
    rank holds the whole FP8 verifier (about 27 GB at the 27B shape) and runs it on
    its own batch row, so there is no pipeline bubble and the hand-off is local.
    The reference's layout (contiguous partitions over ``world - N`` inference
    ranks, nanospec/distributed.py:41-63) remains the default of ``for_world``.
    """

    world: int
    train_gpus: int
    colocate: bool = False
    inference_ranks: list[int] = field(default_factory=list)
    replicate: bool = False

    def __post_init__(self):
        if self.train_gpus not in (1, 2, 4, 8):
            raise ValueError("training ranks must be 1, 2, 4 or 8")
        if self.train_gpus > self.world:
            raise ValueError("more training ranks than GPUs")
        if self.replicate:
            if self.train_gpus != self.world:
                raise ValueError("a replicated verifier needs every GPU to train")
            self.colocate = True
            self.inference_ranks = list(range(self.world))
            return
        if not self.inference_ranks:
            if self.world == self.train_gpus:
                self.colocate = True
                self.inference_ranks = list(range(self.world))
            else:
                self.inference_ranks = list(range(self.train_gpus, self.world))

    @classmethod
    def for_world(cls, world: int, train_gpus: int | None = None) -> "Topology":
        """Default layouts: 8 GPUs -> 4 train + 4 verify; 4 -> 2 + 2; 2 -> 1 + 1; 1 -> colocated."""
        if train_gpus is None:
            train_gpus = {1: 1, 2: 1, 4: 2, 8: 4}.get(world, 1)
        return cls(world=world, train_gpus=train_gpus)

    @classmethod
    def replicated(cls, world: int) -> "Topology":
        """Every GPU trains and holds a full verifier replica."""
        return cls(world=world, train_gpus=world, replicate=True)


def config_path(name: str) -> Path:
    """A config is found by path, else by name in the package's configs/ folder."""
    path = Path(name)
    return path if path.exists() else CONFIG_DIR / f"{name}.json"
