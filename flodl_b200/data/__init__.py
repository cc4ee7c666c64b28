"""Data loading: datasets, samplers, resident/streaming DataLoader with the
staging cascade, fixed-stride record files."""
from .datasets import (CharLM, TokenShards, cifar10, mnist, synthetic_images,  # noqa: F401
                       synthetic_tokens)
from .loader import BatchDataSet, DataLoader, DataLoaderBuilder, DataSet, TensorDataSet  # noqa: F401
from .sampler import (ChunkSampler, DistributedSampler, RandomSampler, Sampler,  # noqa: F401
                      SequentialSampler)
from .records import FixedStrideRecords, RecordDataSet, cifar10_records, mnist_records  # noqa: F401
from .staging import resolve_cached  # noqa: F401
