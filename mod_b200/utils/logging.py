"""Logging with a rank prefix (rank read from RANK when running under torchrun)."""
from __future__ import annotations

import logging
import os


def setup_logging(debug: bool = False, log_file: str = None) -> None:
    rank = os.environ.get("RANK")
    prefix = f"[rank {rank}] " if rank is not None else ""
    fmt = f"%(asctime)s {prefix}%(levelname)s %(name)s: %(message)s"
    handlers = [logging.StreamHandler()]
    if log_file:
        handlers.append(logging.FileHandler(log_file))
    logging.basicConfig(level=logging.DEBUG if debug else logging.INFO, format=fmt, handlers=handlers, force=True)
