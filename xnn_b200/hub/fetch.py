"""Downloaded models: URLs and Zenodo records into a local cache of portable model directories.

``fetch_model(source)`` accepts

* an ``http(s)://`` or ``file://`` URL of a checkpoint file (``.pt`` / ``.pth`` / ``.model``) or of
  an archive (``.zip``, ``.tar``, ``.tar.gz`` / ``.tgz``) holding a portable model directory;
* a Zenodo DOI (``doi:10.5281/zenodo.<id>``, ``https://doi.org/10.5281/zenodo.<id>``) or record
  URL (``https://zenodo.org/records/<id>``): the record's file list comes from the Zenodo REST API
  (``$XNN_B200_ZENODO_API``, default ``https://zenodo.org/api``) and every file is fetched with
  the MD5 the record states.

Files land in one slot per source under :func:`model_cache_dir` and are reused on later calls
(no network then); archives are unpacked in the slot. ``XNN_B200_OFFLINE=1`` turns downloads off.
Parity: the reference's ``fetch_model`` / ``from_pretrained(URL | DOI)``
(``src/xnn/common/models/hub/loader.py:237,414``).
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import shutil
import tarfile
import urllib.request
import zipfile
from pathlib import Path
from typing import List, Optional, Tuple, Union

from ..data.hub.download import fetch, offline

_ZENODO_DOI = re.compile(r"(?:doi:|https?://(?:dx\.)?doi\.org/)?10\.5281/zenodo\.(\d+)$", re.IGNORECASE)
_ZENODO_RECORD = re.compile(r"https?://(?:www\.)?zenodo\.org/(?:records|record)/(\d+)", re.IGNORECASE)
_ARCHIVES = (".zip", ".tar", ".tar.gz", ".tgz")


def model_cache_dir() -> Path:
    v = os.environ.get("XNN_B200_MODELS")
    return Path(v).expanduser() if v else Path.home() / ".cache" / "xnn_b200" / "models"


def is_remote(source) -> bool:
    s = str(source)
    return "://" in s or bool(_ZENODO_DOI.match(s))


def zenodo_record(source: str) -> Optional[str]:
    """The Zenodo record id of a DOI or record URL, or ``None``."""
    for pat in (_ZENODO_DOI, _ZENODO_RECORD):
        m = pat.match(str(source).strip())
        if m:
            return m.group(1)
    return None


def _slot(source: str, cache_dir: Optional[Path]) -> Path:
    base = Path(cache_dir) if cache_dir is not None else model_cache_dir()
    tail = re.sub(r"[^A-Za-z0-9._-]+", "_", source.rstrip("/").split("/")[-1])[:60] or "model"
    digest = hashlib.sha1(source.encode()).hexdigest()[:12]
    return base / f"{tail}-{digest}"


def _record_files(record: str, timeout: float) -> List[Tuple[str, str, Optional[str]]]:
    """``(name, url, md5)`` of every file of a Zenodo record."""
    api = os.environ.get("XNN_B200_ZENODO_API", "https://zenodo.org/api").rstrip("/")
    req = urllib.request.Request(f"{api}/records/{record}", headers={"User-Agent": "xnn_b200",
                                                                     "Accept": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as resp:
        meta = json.load(resp)
    out = []
    for f in meta.get("files", []):
        name = f.get("key") or f.get("filename")
        links = f.get("links", {})
        url = links.get("self") or links.get("download") or links.get("content")
        md5 = None
        cs = f.get("checksum")
        if isinstance(cs, str) and cs.startswith("md5:"):
            md5 = cs[4:]
        if name and url:
            out.append((str(name), str(url), md5))
    if not out:
        raise FileNotFoundError(f"Zenodo record {record} lists no downloadable files")
    return out


def _unpack(path: Path, into: Path) -> None:
    name = path.name.lower()
    if name.endswith(".zip"):
        with zipfile.ZipFile(path) as z:
            for m in z.namelist():
                if os.path.isabs(m) or ".." in Path(m).parts:
                    raise ValueError(f"{path.name}: unsafe member {m!r}")
            z.extractall(into)
    else:
        with tarfile.open(path) as t:
            for m in t.getmembers():
                if os.path.isabs(m.name) or ".." in Path(m.name).parts or m.issym() or m.islnk():
                    raise ValueError(f"{path.name}: unsafe member {m.name!r}")
            t.extractall(into)


def _model_root(slot: Path) -> Path:
    """The portable model directory (or checkpoint file) inside a filled slot."""
    from .card import CARD_FILE, WEIGHTS_FILE
    for marker in (CARD_FILE, WEIGHTS_FILE):
        hits = sorted(slot.rglob(marker))
        if hits:
            return hits[0].parent
    files = sorted(p for p in slot.rglob("*") if p.is_file() and p.suffix in (".pt", ".pth", ".model", ".ckpt"))
    if files:
        return files[0]
    raise FileNotFoundError(f"{slot}: no model directory or checkpoint after the download")


def fetch_model(source: Union[str, Path], cache_dir: Optional[Union[str, Path]] = None, md5: Optional[str] = None,
                timeout: float = 120.0) -> Path:
    """Download ``source`` into the model cache (once) and return the model directory or file."""
    source = str(source)
    slot = _slot(source, Path(cache_dir) if cache_dir is not None else None)
    done = slot / ".complete"
    if done.exists():
        return _model_root(slot)
    if offline():
        raise FileNotFoundError(f"{source} is not in the model cache ({slot}) and downloads are off")
    slot.mkdir(parents=True, exist_ok=True)
    record = zenodo_record(source)
    files = _record_files(record, timeout) if record else [
        (source.split("?")[0].rstrip("/").split("/")[-1] or "model.pt", source, md5)]
    for name, url, sum_ in files:
        dest = fetch(url, slot / name, md5=sum_, timeout=timeout)
        if dest.name.lower().endswith(_ARCHIVES):
            _unpack(dest, slot / (dest.name.split(".")[0] + "_files"))
    root = _model_root(slot)
    done.write_text(source)
    return root


def clear_cache(source: Union[str, Path], cache_dir: Optional[Union[str, Path]] = None) -> None:
    """Remove the cached download of ``source``."""
    slot = _slot(str(source), Path(cache_dir) if cache_dir is not None else None)
    if slot.exists():
        shutil.rmtree(slot)
