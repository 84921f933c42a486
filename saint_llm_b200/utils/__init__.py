"""Utilities: profiling (NVTX ranges behind a flag, device timers with a max over ranks,
throughput / MFU metrics) and failure detection (store-based heartbeats)."""

from saint_llm_b200.utils.heartbeat import Heartbeat, HeartbeatMonitor, stale_ranks
from saint_llm_b200.utils.profiling import DeviceTimer, annotate_blocks, mfu, nvtx_enabled, nvtx_range

__all__ = ["DeviceTimer", "Heartbeat", "HeartbeatMonitor", "annotate_blocks", "mfu", "nvtx_enabled", "nvtx_range",
           "stale_ranks"]
