"""Data: synthetic batches of the benchmark shapes, tar-shard latent datasets, device prefetch."""
from .shards import TarShardDataset, dict_collate, write_shard
from .synthetic import SyntheticWanData
from .prefetch import DevicePrefetcher
from .h3_pool import FileLatentPool

__all__ = ["TarShardDataset", "dict_collate", "write_shard", "SyntheticWanData", "DevicePrefetcher", "FileLatentPool"]
