"""Optimizers and learning-rate schedules."""
from .optimizer import (SGD, Adagrad, Adam, AdamW, NAdam, Optimizer, RAdam, RMSprop,  # noqa: F401
                        migrate_optim_state_file, read_tensor_state, write_tensor_state)
from .scheduler import (CosineScheduler, CyclicLR, ExponentialLR, MultiStepLR, OneCycleLR,  # noqa: F401
                        PlateauScheduler, Scheduler, StepDecay, WarmupScheduler)
