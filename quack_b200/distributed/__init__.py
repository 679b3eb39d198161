"""Multi-GPU overlapped GEMMs: the all-gather runners (``quack.distributed`` in the reference)."""

from .all_gather_gemm import (AllGatherRunner, BlockScaledAllGatherRunner, ring_schedule,  # noqa: F401
                              wait_events_or_report)

__all__ = ["AllGatherRunner", "BlockScaledAllGatherRunner"]
