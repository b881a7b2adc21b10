"""ANI (Smith et al. 2017): element networks on the AEV, with the ANI-1, ANI-1x, ANI-1ccx and
ANI-2x architectures (torchani's per-element widths and self energies, in Hartree) of the
reference (``src/xnn/dnn/models/ani.py:96-358``)."""
from __future__ import annotations

from typing import Optional, Sequence

from ..featurizers.aev import AEV, ANI2X_SPECIES, ANI_SPECIES, angle_shifts, even_shifts
from .descriptor import DescriptorPotential
from .registry import register_model

ANI1X_HIDDEN = {1: (160, 128, 96), 6: (144, 112, 96), 7: (128, 112, 96), 8: (128, 112, 96)}
ANI2X_HIDDEN = {1: (256, 192, 160), 6: (224, 192, 160), 7: (192, 160, 128), 8: (192, 160, 128),
                16: (160, 128, 96), 9: (160, 128, 96), 17: (160, 128, 96)}
ANI1X_SELF_ENERGIES = {1: -0.60095298, 6: -38.08316124, 7: -54.70775770, 8: -75.19446356}
ANI1CCX_SELF_ENERGIES = {1: -0.5991501324919538, 6: -38.03750806057356, 7: -54.67448347695333,
                         8: -75.16043537275567}
ANI2X_SELF_ENERGIES = {1: -0.5978583943827134, 6: -38.08933878049795, 7: -54.71196829862107,
                       8: -75.19106774742086, 16: -398.1577125334925, 9: -99.80348506781634,
                       17: -460.1681939421027}


@register_model("ani")
class ANI(DescriptorPotential):
    def __init__(self, species: Sequence[int] = ANI_SPECIES, radial_cutoff: float = 5.2, angular_cutoff: float = 3.5,
                 hidden=(128, 128, 64), activation="celu", atomic_energies: Optional[Sequence[float]] = None,
                 aev_kwargs: Optional[dict] = None):
        aev = AEV(species, radial_cutoff=radial_cutoff, angular_cutoff=angular_cutoff, **(aev_kwargs or {}))
        super().__init__(aev, species, hidden, activation=activation, atomic_energies=atomic_energies)

    @classmethod
    def ani1(cls, species=ANI_SPECIES, activation="gaussian", atomic_energies=None) -> "ANI":
        return cls(species, 4.6, 3.1, (128, 128, 64), activation, atomic_energies,
                   dict(radial_etas=(16.0,), radial_rs=even_shifts(4.6, 32), angular_etas=(8.0,),
                        angular_zetas=(8.0,), angular_rs=even_shifts(3.1, 8), angular_theta_s=angle_shifts(8)))

    @classmethod
    def ani1x(cls, species=ANI_SPECIES, atomic_energies="torchani") -> "ANI":
        if atomic_energies == "torchani":
            atomic_energies = [ANI1X_SELF_ENERGIES[z] for z in species]
        return cls(species, 5.2, 3.5, {z: ANI1X_HIDDEN[z] for z in species}, "celu", atomic_energies,
                   dict(radial_etas=(16.0,), radial_rs=even_shifts(5.2, 16), angular_etas=(8.0,),
                        angular_zetas=(32.0,), angular_rs=even_shifts(3.5, 4), angular_theta_s=angle_shifts(8)))

    @classmethod
    def ani1ccx(cls, species=ANI_SPECIES, atomic_energies="torchani") -> "ANI":
        if atomic_energies == "torchani":
            atomic_energies = [ANI1CCX_SELF_ENERGIES[z] for z in species]
        return cls.ani1x(species, atomic_energies=atomic_energies)

    @classmethod
    def ani2x(cls, species=ANI2X_SPECIES, atomic_energies="torchani") -> "ANI":
        if atomic_energies == "torchani":
            atomic_energies = [ANI2X_SELF_ENERGIES[z] for z in species]
        return cls(species, 5.1, 3.5, {z: ANI2X_HIDDEN[z] for z in species}, "celu", atomic_energies,
                   dict(radial_etas=(19.7,), radial_rs=even_shifts(5.1, 16, start=0.8), angular_etas=(12.5,),
                        angular_zetas=(14.1,), angular_rs=even_shifts(3.5, 8, start=0.8),
                        angular_theta_s=angle_shifts(4)))

    @classmethod
    def from_config(cls, cfg) -> "ANI":
        extra = dict(cfg.extra or {})
        preset = str(extra.get("preset", "")).lower().replace("_", "-")
        species = [int(z) for z in extra.get("species") or (ANI2X_SPECIES if preset in ("ani-2x", "ani2x")
                                                             else ANI_SPECIES)]
        ae = extra.get("atomic_energies")
        if isinstance(ae, dict):
            ae = [float(ae.get(z, ae.get(str(z), 0.0))) for z in species]
        if preset in ("ani-1", "ani1"):
            return cls.ani1(species, atomic_energies=ae)
        if preset in ("ani-1x", "ani1x"):
            return cls.ani1x(species, atomic_energies="torchani" if ae is None else ae)
        if preset in ("ani-1ccx", "ani1ccx"):
            return cls.ani1ccx(species, atomic_energies="torchani" if ae is None else ae)
        if preset in ("ani-2x", "ani2x"):
            return cls.ani2x(species, atomic_energies="torchani" if ae is None else ae)
        return cls(species, radial_cutoff=float(extra.get("radial_cutoff", cfg.cutoff)),
                   angular_cutoff=float(extra.get("angular_cutoff", min(3.5, cfg.cutoff))),
                   hidden=extra.get("hidden", (128, 128, 64)), activation=extra.get("activation", "celu"),
                   atomic_energies=ae, aev_kwargs=extra.get("aev_kwargs"))
