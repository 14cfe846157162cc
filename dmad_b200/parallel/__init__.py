"""Process groups, data/context parallelism and the fused collective kernels."""
from .dist import (init_distributed, get_rank, get_world_size, is_distributed, barrier, reduce_mean,
                   broadcast_module, max_over_ranks)
from .dp import GradSync

__all__ = ["init_distributed", "get_rank", "get_world_size", "is_distributed", "barrier", "reduce_mean",
           "broadcast_module", "max_over_ranks", "GradSync"]
