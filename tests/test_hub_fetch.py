"""Model downloads through a local HTTP server (127.0.0.1) standing in for a model host and the
Zenodo REST API: archives and single checkpoints, MD5 checks, the cache reused offline."""
import hashlib
import http.server
import json
import os
import shutil
import threading
import zipfile

import pytest
import torch

from xnn_b200.config import from_dict
from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.hub import fetch_model, from_pretrained, register_pretrained, save_pretrained
from xnn_b200.models.registry import prepare_model


@pytest.fixture()
def server(tmp_path):
    root = tmp_path / "www"
    root.mkdir()

    class Handler(http.server.SimpleHTTPRequestHandler):
        def __init__(self, *a, **kw):
            super().__init__(*a, directory=str(root), **kw)

        def log_message(self, *a):
            pass

    httpd = http.server.ThreadingHTTPServer(("127.0.0.1", 0), Handler)
    t = threading.Thread(target=httpd.serve_forever, daemon=True)
    t.start()
    yield root, f"http://127.0.0.1:{httpd.server_address[1]}"
    httpd.shutdown()


def _model_dir(tmp_path):
    cfg = from_dict({"model": {"name": "schnet", "cutoff": 4.0, "n_features": 8, "n_interactions": 1, "n_rbf": 6},
                     "device": "cpu"})
    torch.manual_seed(0)
    model = prepare_model(cfg)
    d = tmp_path / "schnet-small"
    save_pretrained(model, d, config=cfg)
    return model, d


def _energy(model):
    g = collate([structure_to_graph(s, 4.0) for s in synthetic.small_organic(2, seed=4)])
    g.pos = g.pos.to(torch.float32)
    return model(g)["energy"].detach()


def test_archive_url_and_cache(server, tmp_path, monkeypatch):
    root, base = server
    model, d = _model_dir(tmp_path)
    with zipfile.ZipFile(root / "schnet-small.zip", "w") as z:
        for f in d.iterdir():
            z.write(f, f"schnet-small/{f.name}")
    cache = tmp_path / "cache"
    url = f"{base}/schnet-small.zip"
    got = from_pretrained(url, wrap=False, cache_dir=cache)
    torch.testing.assert_close(_energy(got), _energy(model))
    # second use: from the cache, downloads off
    monkeypatch.setenv("XNN_B200_OFFLINE", "1")
    os.remove(root / "schnet-small.zip")
    got2 = from_pretrained(url, wrap=False, cache_dir=cache)
    torch.testing.assert_close(_energy(got2), _energy(model))


def test_zenodo_record_with_checksums(server, tmp_path, monkeypatch):
    root, base = server
    model, d = _model_dir(tmp_path)
    shutil.make_archive(str(root / "bundle"), "gztar", root_dir=str(d.parent), base_dir=d.name)
    data = (root / "bundle.tar.gz").read_bytes()
    api = root / "api" / "records"
    api.mkdir(parents=True)
    meta = {"files": [{"key": "bundle.tar.gz", "links": {"self": f"{base}/bundle.tar.gz"},
                       "checksum": "md5:" + hashlib.md5(data).hexdigest()}]}
    (api / "4242").write_text(json.dumps(meta))
    monkeypatch.setenv("XNN_B200_ZENODO_API", f"{base}/api")
    register_pretrained("schnet-zenodo", "doi:10.5281/zenodo.4242")
    got = from_pretrained("schnet-zenodo", wrap=False, cache_dir=tmp_path / "cache")
    torch.testing.assert_close(_energy(got), _energy(model))
    # a record whose checksum does not match is refused
    meta["files"][0]["checksum"] = "md5:" + "0" * 32
    (api / "4343").write_text(json.dumps(meta))
    with pytest.raises(ValueError, match="MD5"):
        fetch_model("https://doi.org/10.5281/zenodo.4343", cache_dir=tmp_path / "cache2")
