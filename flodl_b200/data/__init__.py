"""Data loading: datasets, samplers, resident/streaming DataLoader."""
from .datasets import (CharLM, TokenShards, cifar10, mnist, synthetic_images,  # noqa: F401
                       synthetic_tokens)
from .loader import BatchDataSet, DataLoader, DataLoaderBuilder, DataSet, TensorDataSet  # noqa: F401
from .sampler import (ChunkSampler, DistributedSampler, RandomSampler, Sampler,  # noqa: F401
                      SequentialSampler)
