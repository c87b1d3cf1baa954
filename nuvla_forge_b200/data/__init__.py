"""Datasets, loaders and the CUDA prefetcher (parity: nuvla_forge/data/__init__.py)."""

from .adapters import REGISTRY, SampleSpec, build_dataset
from .loader import (CudaPrefetcher, LoaderConfig, ShardDataset, SyntheticBatchSource, build_fast_loader,
                     build_naive_loader, describe_environment, normalise_images, write_shards)

__all__ = ["REGISTRY", "CudaPrefetcher", "LoaderConfig", "SampleSpec", "ShardDataset", "SyntheticBatchSource",
           "build_dataset", "build_fast_loader", "build_naive_loader", "describe_environment", "normalise_images",
           "write_shards"]
