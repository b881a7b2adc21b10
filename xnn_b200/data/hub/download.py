"""Cached, MD5-checked file downloads. ``XNN_B200_OFFLINE=1`` (or no network) means: use what is
in the cache, or raise with the path the file is expected at."""
from __future__ import annotations

import hashlib
import os
import urllib.request
from pathlib import Path
from typing import Optional

UNITS = {"kcal_mol_to_ev": 0.0433641153087705, "bohr_to_angstrom": 0.529177210903, "hartree_to_ev": 27.211386245988}


def default_cache_dir() -> Path:
    for var in ("XNN_B200_DATASETS", "XNN_DATASETS", "XNN_CACHE"):
        v = os.environ.get(var)
        if v:
            return Path(v).expanduser()
    return Path.home() / ".cache" / "xnn_b200" / "datasets"


def offline() -> bool:
    return os.environ.get("XNN_B200_OFFLINE", os.environ.get("XNN_OFFLINE", "0")) not in ("0", "", "false")


def md5sum(path: Path, chunk: int = 1 << 20) -> str:
    h = hashlib.md5()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(chunk), b""):
            h.update(block)
    return h.hexdigest()


def fetch(url: str, dest: Path, md5: Optional[str] = None, timeout: float = 60.0) -> Path:
    """``dest`` when it exists (and matches ``md5``), else downloaded from ``url``."""
    dest = Path(dest)
    if dest.exists() and (md5 is None or md5sum(dest) == md5):
        return dest
    if offline():
        raise FileNotFoundError(f"{dest} is not in the dataset cache and downloads are off (XNN_B200_OFFLINE); "
                                f"place the file from {url} there")
    dest.parent.mkdir(parents=True, exist_ok=True)
    tmp = dest.with_name(dest.name + ".part")
    try:
        req = urllib.request.Request(url, headers={"User-Agent": "xnn_b200"})
        with urllib.request.urlopen(req, timeout=timeout) as resp, open(tmp, "wb") as f:
            while True:
                block = resp.read(1 << 20)
                if not block:
                    break
                f.write(block)
    except OSError as err:
        tmp.unlink(missing_ok=True)
        raise FileNotFoundError(f"could not download {url} to {dest} ({err}); place the file there by hand") from err
    if md5 is not None and md5sum(tmp) != md5:
        tmp.unlink(missing_ok=True)
        raise ValueError(f"MD5 mismatch for {dest.name}")
    tmp.replace(dest)
    return dest
