"""Distributed training: DDP tiers, the peer-memory communicator and fused
collectives, ElChe cadence balancing, CPU averaging, outer optimizers."""
from .config import ApplyPolicy, AverageBackend, ElCheConfig, ElCheMode, TrainerConfig  # noqa: F401
from .ddp import Ddp, init_from_env  # noqa: F401
from .outer import NesterovMomentum, OuterAvg, OuterStepper, SlowMomentum, easgd_blend  # noqa: F401
from .trainer import DdpBuilder, DdpHandle, TrainedState, Trainer, Worker  # noqa: F401
