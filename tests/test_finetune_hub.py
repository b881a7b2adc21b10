"""LoRA, multi-head and freezing; portable checkpoints round trip through the hub API."""
import pytest
import torch

from xnn_b200.config import from_dict
from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.registry import prepare_model
from xnn_b200.train.finetune import (MultiHead, count_parameters, freeze_parameters, has_lora, inject_lora,
                                     lora_parameters, merge_lora)


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _cfg(**extra):
    e = {"species": [1, 6, 7, 8, 9, 16, 17], "max_ell": 2, "correlation": 2, "avg_num_neighbors": 6.0}
    e.update(extra)
    return from_dict({"model": {"name": "mace", "cutoff": 4.5, "n_features": 8, "n_interactions": 2, "n_rbf": 6,
                                "extra": e}})


def _batch(n=3, seed=0):
    return collate([structure_to_graph(s, 4.5) for s in synthetic.organic_molecules(n, seed=seed)])


@pytest.mark.parametrize("fast", [False, True])
def test_lora_identity_train_and_merge(fast):
    torch.manual_seed(0)
    m = prepare_model(_cfg()).set_use_fast(fast)
    b = _batch()
    e0 = m(b.clone())["energy"].detach()
    inject_lora(m, rank=2)
    assert has_lora(m)
    torch.testing.assert_close(m(b.clone())["energy"], e0, rtol=1e-12, atol=1e-12)
    trainable = {n for n, p in m.named_parameters() if p.requires_grad}
    assert trainable and all("lora_" in n for n in trainable)
    opt = torch.optim.SGD(list(lora_parameters(m)), lr=1e-2)
    for _ in range(2):
        opt.zero_grad()
        loss = (m(b.clone())["energy"] ** 2).sum()
        loss.backward()
        opt.step()
    e1 = m(b.clone())["energy"].detach()
    assert (e1 - e0).abs().max() > 1e-12
    merge_lora(m)
    assert not has_lora(m)
    torch.testing.assert_close(m(b.clone())["energy"], e1, rtol=1e-10, atol=1e-10)


def test_multihead_matches_single_heads():
    torch.manual_seed(1)
    base = prepare_model(_cfg())
    mh = MultiHead(base, ["pt_head", "Default"])
    with torch.no_grad():
        for p in mh.extra_heads[0].parameters():
            p.add_(0.1 * torch.randn_like(p))
    b = _batch(4, seed=3)
    b.head = torch.tensor([0, 1, 1, 0])
    out = ForceStressOutput(mh)(b.clone())
    h1 = mh.select("Default")
    for h, model in ((0, base), (1, h1)):
        keep = b.head == h
        sub = b.subset(keep)
        ref = ForceStressOutput(model)(sub)
        torch.testing.assert_close(out["energy"][keep], ref["energy"], rtol=1e-10, atol=1e-10)
        node_keep = keep[b.batch]
        torch.testing.assert_close(out["forces"][node_keep], ref["forces"], rtol=1e-9, atol=1e-10)


def test_freeze_parameters():
    m = prepare_model(_cfg())
    total = count_parameters(m)
    left = freeze_parameters(m, freeze=["interactions.*"], trainable=["interactions.0.linear_up.*"])
    assert 0 < left < total
    for n, p in m.named_parameters():
        if n.startswith("interactions.") and not n.startswith("interactions.0.linear_up."):
            assert not p.requires_grad


def test_prepare_model_lora_and_heads_from_config():
    m = prepare_model(_cfg(lora={"rank": 2}, heads=["a", "b"]))
    assert isinstance(m, MultiHead) and has_lora(m)


def test_portable_checkpoint_round_trip(tmp_path):
    from xnn_b200.hub import from_pretrained, load_checkpoint, save_pretrained
    torch.manual_seed(2)
    cfg = _cfg()
    model = ForceStressOutput(prepare_model(cfg))
    b = _batch(2, seed=5)
    ref = model(b.clone())
    out_dir = save_pretrained(model, tmp_path / "my-model", config=cfg)
    ck = load_checkpoint(out_dir)
    assert ck.card.model == "mace" and ck.card.cutoff == 4.5
    again = from_pretrained(out_dir)
    got = again(b.clone())
    torch.testing.assert_close(got["energy"], ref["energy"], rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(got["forces"], ref["forces"], rtol=1e-12, atol=1e-12)
    # a trainer-style checkpoint file converts to a portable directory
    torch.save({"model": model.state_dict(), "cfg": cfg.to_dict()}, tmp_path / "best.pt")
    d2 = save_pretrained(tmp_path / "best.pt", tmp_path / "from-trainer")
    torch.testing.assert_close(from_pretrained(d2)(b.clone())["energy"], ref["energy"], rtol=1e-12, atol=1e-12)


def test_reference_layout_directory_loads(tmp_path):
    """A model directory as the reference writes it: ``model.pt`` holds ``{"model": state_dict}``
    (and a bare state dict, as hand-written directories may hold, loads too)."""
    import yaml

    from xnn_b200.hub import from_pretrained, load_checkpoint
    torch.manual_seed(3)
    cfg = _cfg()
    model = ForceStressOutput(prepare_model(cfg))
    b = _batch(2, seed=6)
    ref = model(b.clone())
    for wrapped in (True, False):
        d = tmp_path / f"ref-layout-{wrapped}"
        d.mkdir()
        sd = {k: v.detach().cpu() for k, v in model.state_dict().items()}
        torch.save({"model": sd} if wrapped else sd, d / "model.pt")
        (d / "config.yaml").write_text(yaml.safe_dump(cfg.to_dict()))
        ck = load_checkpoint(d)
        assert set(ck.state_dict) == set(sd)
        got = from_pretrained(d)(b.clone())
        torch.testing.assert_close(got["energy"], ref["energy"], rtol=1e-12, atol=1e-12)
    # and what this package writes carries the same wrapping
    from xnn_b200.hub import save_pretrained
    out = save_pretrained(model, tmp_path / "ours", config=cfg)
    raw = torch.load(out / "model.pt", weights_only=True)
    assert set(raw) == {"model"} and set(raw["model"]) == set(model.state_dict())
