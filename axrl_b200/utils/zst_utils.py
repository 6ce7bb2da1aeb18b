"""Compressed pickle files with retries (rollout dumps, replay sample sets, mismatch results).

Reference: ``axrl/utils/zst_utils.py:14-58`` (zstd-compressed pickles).  The zstd codec is used
when the ``zstandard`` module is importable; otherwise the payload is zlib-compressed.  The first
four bytes name the codec so either reader can open either file.
"""

from __future__ import annotations

import logging
import pickle
import time
import zlib
from pathlib import Path
from typing import Any

logger = logging.getLogger(__name__)

_ZSTD, _ZLIB = b"AXZS", b"AXZL"


def _codec():  # noqa: ANN202
    try:
        import zstandard  # noqa: F401

        return "zstd"
    except ImportError:
        return "zlib"


def save_zst(obj: Any, path: str | Path, verbose: bool = False, retries: int = 3) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    raw = pickle.dumps(obj, protocol=pickle.HIGHEST_PROTOCOL)
    if _codec() == "zstd":
        import zstandard

        data = _ZSTD + zstandard.ZstdCompressor(level=3).compress(raw)
    else:
        data = _ZLIB + zlib.compress(raw, 3)
    tmp = path.with_suffix(path.suffix + ".tmp")
    for attempt in range(retries):
        try:
            tmp.write_bytes(data)
            tmp.replace(path)  # atomic: a reader never sees a partial file
            break
        except OSError:
            if attempt == retries - 1:
                raise
            time.sleep(0.5 * (attempt + 1))
    if verbose:
        logger.info("saved %s (%.1f MB -> %.1f MB)", path, len(raw) / 1e6, len(data) / 1e6)
    return path


def load_zst(path: str | Path, verbose: bool = False, retries: int = 3) -> Any:
    path = Path(path)
    for attempt in range(retries):
        try:
            data = path.read_bytes()
            break
        except OSError:
            if attempt == retries - 1:
                raise
            time.sleep(0.5 * (attempt + 1))
    head, body = data[:4], data[4:]
    if head == _ZSTD:
        import zstandard

        raw = zstandard.ZstdDecompressor().decompress(body)
    elif head == _ZLIB:
        raw = zlib.decompress(body)
    else:
        raise ValueError(f"{path}: not a compressed pickle written by save_zst")
    if verbose:
        logger.info("loaded %s", path)
    return pickle.loads(raw)  # noqa: S301 - files written by this framework
