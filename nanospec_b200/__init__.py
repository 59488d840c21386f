"""nanospec_b200: a Blackwell-native (sm_100a) speculative-draft training runtime.

Hand-written forward and backward for every op (no autograd), CUDA kernels for
B200 on the GPU path, NCCL plus peer-memory kernels for communication.
"""

from .config import DraftConfig, Objective, Topology, config_path
from .data import PreparedBatch, prepare, sample_anchors
from .engine import TrainResult, train
from .models.draft import DSpark, initialize, parameter_shapes
from .objective import LossMetrics
from .parallel.node import Node, TeacherBatch
from .parallel.optim import AdamW, adamw_step, zero_grad

__all__ = [
    "AdamW", "DSpark", "DraftConfig", "LossMetrics", "Node", "Objective", "PreparedBatch",
    "TeacherBatch", "Topology", "TrainResult", "adamw_step", "config_path", "initialize",
    "parameter_shapes", "prepare", "sample_anchors", "train", "zero_grad",
]
