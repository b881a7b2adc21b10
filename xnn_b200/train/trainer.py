"""``Trainer(cfg, train, val, test).fit()`` -- energy/force/stress training on one or many GPUs.

Behaviour follows the reference trainer (``src/xnn/common/train/trainer.py:237-1441``):
the model comes from :func:`~xnn_b200.models.prepare_model` wrapped in
:class:`~xnn_b200.models.ForceStressOutput` (forces / stress only when their loss weight
is positive); the validation and test sets are seeded random splits when not given;
training shards with a distributed sampler, evaluation with strided shards; Adam / AMSGrad
/ AdamW with a plateau or cosine schedule, an optional float64 EMA of the weights, and
rank 0 writes ``best.pt`` (on monitor improvement) and ``last.pt`` as
``{"model": state_dict, "cfg": config dict}`` with the ``ForceStressOutput`` key layout.

The step is built for the GPU:

* gradients live in one flat buffer (:class:`~xnn_b200.parallel.grad_sync.GradSync`); the
  data-parallel reduction is one collective on it (NCCL, or the fused peer-to-peer
  kernel with ``trainer.grad_sync = "p2p"``);
* the force pass and the parameter pass tell the fused kernels which derivatives are
  unused (:mod:`xnn_b200.ops.modes`), so neither forms parameter gradients in the force
  pass nor geometric cotangents in the parameter pass;
* with ``trainer.cuda_graph`` the whole step -- forward, force pass, loss, double backward,
  all-reduce, optimizer and EMA -- is one CUDA graph over padded fixed-capacity batches
  (:mod:`xnn_b200.train.graphed`); nothing in the step synchronises with the host.
"""
from __future__ import annotations

import math
import os
import time
from typing import Dict, List, Optional, Sequence

import torch
from torch import Tensor, nn

from ..data import AtomicGraph, collate
from ..models import ForceStressOutput, prepare_model
from ..ops.modes import params_only
from ..parallel import distributed as D
from ..parallel.grad_sync import GradSync
from .graphed import GraphedStep, PaddedCollate, batch_sizes
from .losses import error_metrics, weighted_loss


class EMA:
    """Float64 shadow of the trainable weights, ``s <- d s + (1 - d) w`` after every step."""

    def __init__(self, params: Sequence[nn.Parameter], decay: float):
        self.params = list(params)
        self.decay = float(decay)
        self.shadow = [p.detach().to(torch.float64).clone() for p in self.params]

    @torch.no_grad()
    def update(self) -> None:
        w = [p.detach().to(torch.float64) for p in self.params]
        torch._foreach_mul_(self.shadow, self.decay)
        torch._foreach_add_(self.shadow, w, alpha=1.0 - self.decay)

    @torch.no_grad()
    def swap(self) -> None:
        for p, s in zip(self.params, self.shadow):
            tmp = p.detach().clone()
            p.copy_(s.to(p.dtype))
            s.copy_(tmp.to(torch.float64))


def _random_split(n: int, fractions, seed: int):
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n, generator=g).tolist()
    out, start = [], 0
    for f in fractions:
        k = int(round(f * n))
        out.append(perm[start:start + k])
        start += k
    out.append(perm[start:])
    return out


class _Subset(torch.utils.data.Dataset):
    def __init__(self, base, idx):
        self.base, self.idx = base, list(idx)

    def __len__(self):
        return len(self.idx)

    def __getitem__(self, i):
        return self.base[self.idx[i]]


class Trainer:
    def __init__(self, cfg, train, val=None, test=None, model: Optional[nn.Module] = None,
                 replay_set=None, callbacks: Optional[list] = None, loggers: Optional[list] = None,
                 reactions=None, val_reactions=None):
        self.cfg = cfg
        dev_req = cfg.device
        self.device = D.init_process_group(None if dev_req == "auto" else dev_req)
        self.rank, self.world = D.rank(), D.world_size()
        torch.manual_seed(cfg.seed)
        base = model if model is not None else prepare_model(cfg)
        o = cfg.optim
        self.module = ForceStressOutput(base, compute_forces=o.force_weight > 0,
                                        compute_stress=o.stress_weight > 0).to(self.device)
        self.module.train()
        self._freeze()
        self.params = [p for p in self.module.parameters() if p.requires_grad]
        backend = cfg.trainer.grad_sync
        if backend == "auto":
            backend = "nccl"
        self._grad_backend = backend if self.world > 1 else "none"
        self.grad_sync = GradSync(self.params, backend=self._grad_backend)
        # same starting weights on every rank
        if self.world > 1:
            with torch.no_grad():
                for t in list(self.module.parameters()) + list(self.module.buffers()):
                    torch.distributed.broadcast(t, 0)
        graphs = bool(cfg.trainer.cuda_graph) and self.device.type == "cuda"
        self.use_graphs = graphs
        lr = torch.tensor(o.lr, device=self.device) if graphs else o.lr
        opt_kw = dict(lr=lr, weight_decay=o.weight_decay)
        if self.device.type == "cuda":
            opt_kw.update(fused=True, capturable=graphs)
        name = o.optimizer.lower()
        if name == "adamw":
            self.optimizer = torch.optim.AdamW(self.params, **opt_kw)
        elif name in ("adam", "amsgrad"):
            self.optimizer = torch.optim.Adam(self.params, amsgrad=name == "amsgrad", **opt_kw)
        else:
            raise ValueError(f"unknown optimizer {o.optimizer!r}")
        if o.scheduler == "cosine":
            self.scheduler = torch.optim.lr_scheduler.CosineAnnealingLR(self.optimizer, T_max=max(1, o.epochs),
                                                                        eta_min=o.min_lr)
        elif o.scheduler == "plateau":
            self.scheduler = torch.optim.lr_scheduler.ReduceLROnPlateau(
                self.optimizer, mode=cfg.trainer.mode, factor=o.plateau_factor,
                patience=o.plateau_patience, min_lr=o.min_lr)
        else:
            self.scheduler = None
        self.ema = EMA(self.params, o.ema_decay) if o.ema_decay > 0 else None
        self.loss_weights = self._make_loss_weights(o)
        self._fused = None
        fs = cfg.trainer.fused_step
        if self.loss_weights is not None and fs is True:
            raise ValueError("trainer.fused_step computes fixed-weight losses; optim.loss_weighting: uncertainty "
                             "runs in the ordinary step")
        if self.loss_weights is None and (fs is True or (fs == "auto" and self.device.type == "cuda")):
            from . import mace_step
            ok, why = mace_step.supports(self.module, o)
            if ok:
                self._fused = mace_step.MACEStep(self.module, o.energy_weight, o.force_weight)
                # the flat gradient buffer in the step's bucket order (interaction by interaction)
                self.grad_sync.close()
                self.grad_sync = GradSync(self.params, backend=self._grad_backend,
                                          buckets=self._fused.bucket_params())
            elif fs is True:
                raise ValueError(f"trainer.fused_step: {why}")
        self.train_set, self.val_set, self.test_set = self._splits(train, val, test)
        self.callbacks = list(callbacks or [])
        from .loggers import make_loggers
        self.loggers = loggers if loggers is not None else (make_loggers(cfg) if D.is_main() else [])
        self._graphed: Optional[GraphedStep] = None
        self._setup_reactions(reactions, val_reactions)
        self._padder: Optional[PaddedCollate] = None
        self.epoch = 0
        self.global_step = 0
        self.best = None
        self.history: List[Dict[str, float]] = []

    # ------------------------------------------------------------------ setup
    def _make_loss_weights(self, o):
        """:class:`UncertaintyWeights` over the active loss terms (``optim.loss_weighting:
        uncertainty``, ordinary single-head steps), their ``log sigma`` in the optimizer without
        weight decay; ``None`` for fixed weights."""
        if o.loss_weighting not in ("fixed", "uncertainty"):
            raise ValueError(f"optim.loss_weighting must be 'fixed' or 'uncertainty', got {o.loss_weighting!r}")
        if o.loss_weighting == "fixed":
            return None
        if self.use_graphs:
            raise ValueError("optim.loss_weighting: uncertainty does not run in captured steps (trainer.cuda_graph)")
        from .losses import LOSS_TERMS, UncertaintyWeights
        names = [n for n, w in LOSS_TERMS.items() if getattr(o, w, 0.0) > 0]
        if not names:
            raise ValueError("optim.loss_weighting: uncertainty needs a loss term with a positive weight")
        uw = UncertaintyWeights(names).to(self.device, self.params[0].dtype)
        if self.world > 1:
            with torch.no_grad():
                for p in uw.parameters():
                    torch.distributed.broadcast(p, 0)
        self.optimizer.add_param_group({"params": list(uw.parameters()), "weight_decay": 0.0})
        return uw

    def _freeze(self):
        import fnmatch
        o = self.cfg.optim
        for name, p in self.module.named_parameters():
            if o.train_only and not any(fnmatch.fnmatch(name, pat) or pat in name for pat in o.train_only):
                p.requires_grad_(False)
            if any(fnmatch.fnmatch(name, pat) or pat in name for pat in o.freeze):
                p.requires_grad_(False)

    def _splits(self, train, val, test):
        d = self.cfg.data
        if val is None and d.val_fraction > 0 or test is None and d.test_fraction > 0:
            fr = []
            if val is None:
                fr.append(d.val_fraction)
            if test is None:
                fr.append(d.test_fraction)
            parts = _random_split(len(train), fr, self.cfg.seed)
            i = 0
            if val is None:
                val = _Subset(train, parts[i]); i += 1
            if test is None:
                test = _Subset(train, parts[i]); i += 1
            train = _Subset(train, parts[-1])
        return train, val, test

    # ------------------------------------------------------------------ reactions
    def _setup_reactions(self, reactions, val_reactions) -> None:
        """Reaction sets (``xnn_b200.train.reactions.ReactionSet``): with ``optim.reaction_weight > 0``
        each step adds the loss of ``optim.reaction_batch_size`` reactions, drawn in turn from a
        shuffled order; ``val_reactions`` are scored at every validation."""
        o = self.cfg.optim
        self.reactions, self.val_reactions, self._reaction_batches = reactions, val_reactions, None
        if o.reaction_weight > 0:
            if reactions is None or len(reactions) == 0:
                raise ValueError("optim.reaction_weight > 0 needs reactions (a ReactionSet)")
            if self.use_graphs or self.world > 1:
                raise ValueError("the reaction-energy term runs in ordinary single-process steps "
                                 "(trainer.cuda_graph off, one process)")
            if o.reaction_batch_size < 1:
                raise ValueError(f"optim.reaction_batch_size must be positive, got {o.reaction_batch_size}")

    def _next_reactions(self):
        if self._reaction_batches is None:
            def endless():
                epoch = 0
                while True:
                    yield from self.reactions.batches(self.cfg.optim.reaction_batch_size, True, self.cfg.seed + epoch)
                    epoch += 1
            self._reaction_batches = endless()
        return next(self._reaction_batches)

    def _reaction_loss(self, rs) -> Tensor:
        o = self.cfg.optim
        base = self.module.model
        e = rs.species_energies(base, float(self.cfg.model.cutoff), device=self.device)
        delta = o.huber_delta if o.huber_delta_reactions is None else o.huber_delta_reactions
        return rs.loss(e, delta)

    # ------------------------------------------------------------------ step
    def _loss(self, batch: AtomicGraph):
        o = self.cfg.optim
        out = self.module(batch)
        learned = self.loss_weights is not None and self.module.training
        parts = {} if learned else None
        loss, logs = weighted_loss(out, batch, o.energy_weight, o.force_weight, o.stress_weight,
                                   dipole_weight=o.dipole_weight,
                                   polarizability_weight=o.polarizability_weight,
                                   charge_weight=o.charge_weight, property_weight=o.property_weight,
                                   huber_delta=o.huber_delta, huber_delta_energy=o.huber_delta_energy,
                                   huber_delta_forces=o.huber_delta_forces,
                                   huber_delta_stress=o.huber_delta_stress, parts=parts)
        if learned:
            loss = self.loss_weights(parts)
            logs = dict(logs, **{f"sigma_{k}": torch.exp(p.detach()) for k, p in self.loss_weights.log_sigma.items()})
        if o.reaction_weight > 0 and self.module.training and self.reactions is not None and not self.use_graphs:
            r = self._reaction_loss(self._next_reactions())
            loss = loss + o.reaction_weight * r.to(loss.dtype)
            logs = dict(logs, reaction=r.detach())
        return loss, logs, out

    def _train_step_impl(self, batch: AtomicGraph):
        self.grad_sync.zero_()
        if self.loss_weights is not None:
            for p in self.loss_weights.parameters():
                p.grad = None
        if self._fused is not None:
            loss, logs, _ = self._fused(batch, bucket_hook=self.grad_sync.bucket_ready)
        else:
            loss, logs, _ = self._loss(batch)
            with params_only():
                inputs = self.params if self.loss_weights is None else self.params + list(
                    self.loss_weights.parameters())
                loss.backward(inputs=inputs)
        self.grad_sync.reduce()
        if self.loss_weights is not None and self.world > 1:
            for p in self.loss_weights.parameters():
                torch.distributed.all_reduce(p.grad)
                p.grad.mul_(1.0 / self.world)
        if self.cfg.optim.clip_grad > 0:
            torch.nn.utils.clip_grad_norm_(self.params, self.cfg.optim.clip_grad, foreach=True)
        self.optimizer.step()
        if self.ema is not None:
            self.ema.update()
        return loss.detach(), {k: v.detach() for k, v in logs.items()}

    def capacity_for(self, datasets, batch_size: int, headroom: Optional[float] = None):
        """Padding capacities covering batches of ``batch_size`` structures from ``datasets``."""
        h = self.cfg.trainer.graph_headroom if headroom is None else headroom
        sizes = []
        for ds in datasets:
            for i in range(len(ds)):
                g = ds[i]
                sizes.append((g.num_nodes, g.num_edges))
        sizes.sort(key=lambda t: -t[0])
        top = sizes[:batch_size]
        n = sum(s[0] for s in top)
        es = sorted((s[1] for s in sizes), reverse=True)[:batch_size]
        e = sum(es)
        return int(n * (1 + h)) + 2, int(e * (1 + h)) + 1, batch_size + 1

    def capacity_for_batches(self, batches, headroom: Optional[float] = None):
        """Padding capacities covering the given batches (lists of graphs, or collated graphs).

        Sizing the captured step to the batches a run actually draws (instead of the worst case
        of any ``batch_size`` structures) keeps the padded work close to the real work."""
        h = self.cfg.trainer.graph_headroom if headroom is None else headroom
        n = e = g = 0
        for b in batches:
            if isinstance(b, (list, tuple)):
                n = max(n, sum(x.num_nodes for x in b))
                e = max(e, sum(x.num_edges for x in b))
                g = max(g, len(b))
            else:
                n, e, g = max(n, b.num_nodes), max(e, b.num_edges), max(g, b.num_graphs)
        return int(n * (1 + h)) + 2, int(e * (1 + h)) + 1, g + 1

    def make_padder(self, max_atoms: int, max_edges: int, max_graphs: int) -> PaddedCollate:
        self._padder = PaddedCollate(max_atoms, max_edges, max_graphs, self.cfg.model.cutoff,
                                     pin_memory=self.device.type == "cuda")
        return self._padder

    def train_step(self, batch: AtomicGraph):
        """One optimisation step on ``batch`` (host or device); returns ``(loss, logs)`` tensors.

        With ``trainer.cuda_graph`` the batch must be padded by :meth:`make_padder`'s collate;
        the first call captures the step.
        """
        self.module.train()
        if self.use_graphs:
            if self._graphed is None:
                self._graphed = GraphedStep(self._train_step_impl, batch, self.device)
            out = self._graphed(batch)
        else:
            out = self._train_step_impl(batch.to(self.device, non_blocking=True))
        self.global_step += 1
        # a fused all-reduce that timed out left the ranks with different gradients: stop here
        # (host-mapped status, no synchronisation; it reports the steps finished so far)
        self.grad_sync.check()
        return out

    # ------------------------------------------------------------------ data
    def _loader(self, ds, train: bool):
        from torch.utils.data import DataLoader
        d = self.cfg.data
        if ds is None or len(ds) == 0:
            return None
        if train:
            sampler = torch.utils.data.distributed.DistributedSampler(
                ds, num_replicas=self.world, rank=self.rank, shuffle=d.shuffle,
                seed=self.cfg.seed, drop_last=self.use_graphs) if self.world > 1 else None
            shuffle = d.shuffle and sampler is None
        else:
            idx = D.shard_indices(len(ds))
            ds = _Subset(ds, idx)
            sampler, shuffle = None, False
        col = collate
        if train and self.use_graphs:
            if self._padder is None:
                self.make_padder(*self.capacity_for([ds], d.batch_size))
            col = self._padder
        g = torch.Generator().manual_seed(self.cfg.seed + self.rank)
        return DataLoader(ds, batch_size=d.batch_size, shuffle=shuffle, sampler=sampler,
                          collate_fn=col, num_workers=d.num_workers, generator=g,
                          drop_last=train and self.use_graphs,
                          pin_memory=False, persistent_workers=d.num_workers > 0)

    # ------------------------------------------------------------------ loop
    def evaluate(self, ds, prefix: str = "val") -> Dict[str, float]:
        loader = self._loader(ds, train=False)
        if loader is None:
            return {}
        was = self.module.training
        self.module.train()  # the force loss needs the graph of forces in train mode
        if self.ema is not None:
            self.ema.swap()
        tot: Dict[str, Tensor] = {}
        loss_sum = torch.zeros((), dtype=torch.float64, device=self.device)
        n_batches = torch.zeros((), dtype=torch.float64, device=self.device)
        for batch in loader:
            batch = batch.to(self.device)
            loss, logs, out = self._loss(batch)
            loss_sum += loss.detach().to(torch.float64)
            n_batches += 1
            for k, v in error_metrics(out, batch).items():
                tot[k] = tot.get(k, 0) + v.to(torch.float64)
        if self.ema is not None:
            self.ema.swap()
        self.module.train(was)
        keys = sorted(tot)
        vec = torch.stack([loss_sum, n_batches] + [tot[k] for k in keys])
        D.all_reduce_sum(vec)
        vals = vec.tolist()
        res = {f"{prefix}/loss": vals[0] / max(vals[1], 1.0)}
        if prefix == "val" and self.val_reactions is not None and len(self.val_reactions):
            with torch.no_grad():
                e = self.val_reactions.species_energies(self.module.model, float(self.cfg.model.cutoff),
                                                        device=self.device)
                err = self.val_reactions.errors(e)
                res["val/reaction_mae"] = float(err.abs().mean())
                res["val/reaction_rmse"] = float(err.pow(2).mean().sqrt())
                res["val/reaction_mse"] = float(self.val_reactions.loss(e))
        got = dict(zip(keys, vals[2:]))
        for q in ("energy", "forces", "stress"):
            if f"{q}_n" in got and got[f"{q}_n"] > 0:
                res[f"{prefix}/{q}_mae"] = got[f"{q}_abs"] / got[f"{q}_n"]
                res[f"{prefix}/{q}_rmse"] = math.sqrt(got[f"{q}_sq"] / got[f"{q}_n"])
        return res

    def _train_epoch(self) -> Dict[str, float]:
        loader = self._loader(self.train_set, train=True)
        if hasattr(loader.sampler, "set_epoch"):
            loader.sampler.set_epoch(self.epoch)
        loss_sum = torch.zeros((), dtype=torch.float64, device=self.device)
        n = 0
        for batch in loader:
            loss, _ = self.train_step(batch)
            loss_sum += loss.to(torch.float64)
            n += 1
            for cb in self.callbacks:
                cb.on_train_batch_end(self, loss)
        t = torch.stack([loss_sum, torch.tensor(float(n), dtype=torch.float64, device=self.device)])
        D.all_reduce_sum(t)
        out = {"train/loss": float(t[0] / t[1].clamp_min(1.0))}
        self.grad_sync.check()         # every step of the epoch has finished (synchronised above)
        return out

    def fit(self) -> Dict[str, float]:
        from .callbacks import ModelCheckpoint
        tcfg = self.cfg.trainer
        if not any(isinstance(c, ModelCheckpoint) for c in self.callbacks):
            self.callbacks.append(ModelCheckpoint(self.cfg.output_dir, tcfg.monitor, tcfg.mode,
                                                  tcfg.save_every_n_epochs))
        for cb in self.callbacks:
            cb.on_fit_start(self)
        metrics: Dict[str, float] = {}
        try:
            for epoch in range(self.cfg.optim.epochs):
                self.epoch = epoch
                t0 = time.perf_counter()
                metrics = self._train_epoch()
                if self.val_set is not None and len(self.val_set) and (epoch + 1) % tcfg.val_every_n_epochs == 0:
                    metrics.update(self.evaluate(self.val_set, "val"))
                metrics["epoch"] = epoch
                metrics["time_s"] = time.perf_counter() - t0
                metrics["lr"] = float(self.optimizer.param_groups[0]["lr"])
                if self.scheduler is not None:
                    if isinstance(self.scheduler, torch.optim.lr_scheduler.ReduceLROnPlateau):
                        self.scheduler.step(metrics.get(tcfg.monitor, metrics["train/loss"]))
                    else:
                        self.scheduler.step()
                self.history.append(dict(metrics))
                if (epoch + 1) % tcfg.log_every_n_epochs == 0:
                    for lg in self.loggers:
                        lg.log(metrics, step=epoch)
                stop = False
                for cb in self.callbacks:
                    stop |= bool(cb.on_epoch_end(self, metrics))
                if stop:
                    break
            if self.test_set is not None and len(self.test_set):
                metrics.update(self.evaluate(self.test_set, "test"))
        finally:
            for cb in self.callbacks:
                cb.on_fit_end(self)
            for lg in self.loggers:
                lg.close()
        return metrics

    # ------------------------------------------------------------------ checkpoints
    def state_dict_for_save(self) -> Dict[str, Tensor]:
        if self.ema is not None:
            self.ema.swap()
        sd = {k: v.detach().cpu().clone() for k, v in self.module.state_dict().items()}
        if self.ema is not None:
            self.ema.swap()
        return sd

    def save(self, path: str) -> None:
        if D.is_main():
            os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
            state = {"model": self.state_dict_for_save(), "cfg": self.cfg.to_dict()}
            if self.loss_weights is not None:
                state["loss_sigmas"] = self.loss_weights.sigmas()
            torch.save(state, path)
        D.barrier()

    def close(self) -> None:
        if self._graphed is not None:
            self._graphed.release()
            self._graphed = None
        self.grad_sync.close()
