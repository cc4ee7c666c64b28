"""Neural-network modules, losses, initialisers, AMP, CUDA graphs, checkpoints."""
from . import init  # noqa: F401
from .activation import (ELU, GELU, SELU, GeluApprox, Hardsigmoid, Hardswish, LeakyReLU,  # noqa: F401
                         LogSoftmax, Mish, PReLU, ReLU, Sigmoid, SiLU, Softmax, Softplus, SwiGLU,
                         Tanh)
from .amp import (AutocastGuard, GradScaler, autocast, cast_parameters,  # noqa: F401
                  is_autocast_enabled, is_autocast_enabled_for)
from .checkpoint import (LoadReport, MigrateReport, checkpoint_keys, checkpoint_version,  # noqa: F401
                         load_checkpoint, load_checkpoint_file, load_model, migrate_checkpoint,
                         migrate_checkpoint_file, read_checkpoint, save_checkpoint,
                         save_checkpoint_file, save_model)
from .clip import clip_grad_norm, clip_grad_value  # noqa: F401
from .cuda_graph import CaptureMode, GpuGraph, MemPoolId, gpu_graph_capture, gpu_graph_pool_handle  # noqa: F401
from .layers import (AdaptiveAvgPool2d, AdaptiveMaxPool2d, AlphaDropout, AvgPool1d,  # noqa: F401
                     AvgPool2d, BatchNorm, BatchNorm2d, Bilinear, Conv1d, Conv2d, Conv3d,
                     ConvTranspose1d, ConvTranspose2d, ConvTranspose3d, Dropout, Dropout2d,
                     Embedding, EmbeddingBag, Flatten, Fold, GaussianBlur, GroupNorm, GRU, GRUCell,
                     Identity, InstanceNorm, LayerNorm, Linear, LSTM, LSTMCell, MaxPool1d,
                     MaxPool2d, MultiheadAttention, PixelShuffle, PixelUnshuffle, ReflectionPad2d,
                     RMSNorm, RotaryEmbedding, Unfold, Upsample, ZeroPad2d, gaussian_blur_2d)
from .loss import (bce_loss, bce_with_logits_loss, cosine_embedding_loss, cross_entropy_loss,  # noqa: F401
                   ctc_loss, focal_loss, hinge_embedding_loss, kl_div_loss, l1_loss,
                   margin_ranking_loss, mse_loss, nll_loss, poisson_nll_loss, smooth_l1_loss,
                   triplet_margin_loss)
from .module import Module, NamedInputModule, walk_modules  # noqa: F401
from ..optim import (SGD, Adagrad, Adam, AdamW, CosineScheduler, CyclicLR, ExponentialLR,  # noqa: F401
                     MultiStepLR, NAdam, OneCycleLR, Optimizer, PlateauScheduler, RAdam, RMSprop,
                     Scheduler, StepDecay, WarmupScheduler, migrate_optim_state_file)
