"""Fused op layer: autograd Functions over the sm_100a kernel library."""
from .attention import attention_packed, scaled_dot_product_attention  # noqa: F401
from .linear import linear  # noqa: F401
from .loss import cross_entropy  # noqa: F401
from .misc import (batch_norm2d, conv1d, conv2d, conv_transpose1d, conv_transpose2d,  # noqa: F401
                   dropout, embedding, gelu, max_pool1d, max_pool2d)
from .norm import group_norm, layer_norm, rms_norm  # noqa: F401
from .transformer import lm_train_loss  # noqa: F401,E402
from .bert import bert_mlm_train_loss  # noqa: F401,E402
from .resnet import resnet_train_loss  # noqa: F401,E402
