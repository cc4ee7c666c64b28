"""flodl_b200: a B200-native deep-learning framework with floDl's capabilities.

Layers: ``tensor`` helpers over libtorch tensors/autograd, ``ops`` (sm_100a
kernels behind autograd), ``nn`` (modules, losses, AMP, CUDA graphs,
checkpoints), ``optim``, ``graph`` (FlowBuilder, graph trees), ``data``,
``parallel`` (DDP, fused peer-memory collectives, ElChe trainer), ``monitor``,
``hf`` (HuggingFace loading) and ``models``.
"""
__version__ = "0.1.0"

from . import nn, ops, optim  # noqa: F401,E402
from .graph import FlowBuilder, Graph, MergeOp  # noqa: F401,E402
from .tensor import Device, manual_seed, no_grad, test_device  # noqa: F401,E402
