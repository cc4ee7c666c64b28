"""Distributed training: DDP tiers, the peer-memory communicator and fused
collectives, ElChe cadence balancing with the LR-aware meta-controller, CPU
averaging (controller, client, per-host relay), outer optimizers, the
distributed runtime (rendezvous, membership, launcher, dial-in agents, port
mux and status board, cluster topology), coordinator pieces, the NCCL
communicator layer and checkpoint bundles."""
from .bundle import (CheckpointBundle, CheckpointForge, CheckpointMeta, RankDeathRecord,  # noqa: F401
                     SaveReason, load_bundle, save_bundle)
from .cluster import (ClusterBuilder, FullCluster, LocalCluster, discover_test_cluster,  # noqa: F401
                      model_sig, module_sig)
from .config import ApplyPolicy, AverageBackend, ElCheConfig, ElCheMode, TrainerConfig  # noqa: F401
from .coordinator import (AlertLane, CallbackRoles, ChunkPool, MaxFailureThreshold,  # noqa: F401
                          WindowLedger)
from .ddp import Ddp, init_from_env  # noqa: F401
from .launcher import LocalLauncher, Role, init_rank, role_from_env  # noqa: F401
from .membership import ClusterPhase, JoinWindow, StartMode  # noqa: F401
from .meta import LrEventMeta  # noqa: F401
from .outer import NesterovMomentum, OuterAvg, OuterStepper, SlowMomentum, easgd_blend  # noqa: F401
from .trainer import DdpBuilder, DdpHandle, TrainedState, Trainer, Worker  # noqa: F401
