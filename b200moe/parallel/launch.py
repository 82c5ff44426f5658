"""Helpers for externally launched (torchrun) multi-GPU runs."""
from __future__ import annotations

import os
import time


def _addr():
    return os.environ.get("MASTER_ADDR", "127.0.0.1"), int(os.environ.get("MASTER_PORT", "29500")) + 1


def driver_store():
    """Rank 0 of a torchrun job: host the store the idle ranks poll."""
    import torch.distributed as dist
    from datetime import timedelta
    host, port = _addr()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    return dist.TCPStore(host, port, world, True, timeout=timedelta(seconds=3600), wait_for_workers=False)


def wait_for_driver(poll_s: float = 1.0) -> int:
    """Non-driver torchrun ranks: stay alive without touching CUDA until the
    driver (rank 0) finishes; the driver's engine spawns the per-GPU workers.
    Returns when the TCP store says the driver is done (or it disappears)."""
    import torch.distributed as dist
    from datetime import timedelta
    host, port = _addr()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    store = dist.TCPStore(host, port, world, False, timeout=timedelta(seconds=3600))
    while True:
        try:
            if store.check(["driver_done"]):
                return 0
        except Exception:
            return 0
        time.sleep(poll_s)
