"""Dataset builders: published sets read from their distribution files (rMD17, QM7), sets that
ship as files (argon MD, any extxyz / RuNNer file) and the seeded synthetic benchmark sets."""
from __future__ import annotations

from pathlib import Path
from typing import Optional

import numpy as np

from .base import DatasetBuilder, register_dataset, select_split
from .download import UNITS, fetch

_FIGSHARE = "https://ndownloader.figshare.com/files/{}"
# rMD17 (Christensen & von Lilienfeld 2020): figshare file ids and MD5 sums of the molecule archives
_RMD17 = {"aspirin": ("62265757", "17fd6fb69066888613f7e16b358a7553"),
          "azobenzene": ("62265754", "be79df918468eb3579aa73a0becf7390"),
          "benzene": ("62265739", "18c9242bc90fbf28215f6dd81e650f16"),
          "ethanol": ("62265733", "eb837fb8deb27d4e0d52f71a03aff776"),
          "malonaldehyde": ("62265736", "cdc1d70c0c34062ddde6e5071eb6fe21"),
          "naphthalene": ("62265751", "0efba19c9907e3852318b1e6008b3b9e"),
          "paracetamol": ("62265760", "ba10784f7b67635427085f6d7ec2dd97"),
          "salicylic": ("62265748", "900fedf242da438400fa4293348d7dd1"),
          "toluene": ("62265742", "0f2913d51f8149c90ab28d697a076f64"),
          "uracil": ("62265745", "992a4479c28a07e0cce6da964805be31")}
_RMD17_SPLITS = {("train", 1): ("62265793", "22264dcf2e42d6133362411abbbe4ce8"),
                 ("train", 2): ("62265772", "28dbc9a3d5e7c47e653b1cc01809df35"),
                 ("train", 3): ("62265775", "8de68b1b288c790e633c9d05ff5f04dd"),
                 ("train", 4): ("62265766", "3764257abf8121a0905f364468ba83da"),
                 ("train", 5): ("62265778", "4670362bd554c9c22581c936432236b3"),
                 ("test", 1): ("62265781", "124c8a0849e84e244d6ce8424e1c05cf"),
                 ("test", 2): ("62265769", "9dc098724c1680daca038b785ee4f602"),
                 ("test", 3): ("62265787", "fd96f4623291dc23dd80b24dd634ca0b"),
                 ("test", 4): ("62265790", "f0acce759fa4fe46b3a0b2a450e7e260"),
                 ("test", 5): ("62265784", "4892da12e88a3c30c9a15f1f95e6eaac")}
_QM7 = ("http://quantum-machine.org/data/qm7.mat", "2aea1a6ac88793faeafcd61a2491f059")


class RMD17(DatasetBuilder):
    name = "rmd17"
    description = "Revised MD17: 10 small molecules, PBE/def2-SVP energies and forces (eV, A by default)."

    def load(self, *, split=None, cache_dir: Path, molecule: Optional[str] = None, fold: int = 1, units: str = "eV",
             n_train: Optional[int] = None, n_test: Optional[int] = None):
        if molecule is None:
            raise ValueError("rmd17 needs `molecule`: one of " + ", ".join(sorted(_RMD17)))
        mol = {"salicylic_acid": "salicylic", "salicylic acid": "salicylic"}.get(molecule.lower(), molecule.lower())
        if mol not in _RMD17:
            raise ValueError(f"unknown rmd17 molecule {molecule!r}; choose one of " + ", ".join(sorted(_RMD17)))
        if units not in ("eV", "kcal/mol", "kcal"):
            raise ValueError(f"units must be 'eV' or 'kcal/mol', got {units!r}")
        root = Path(cache_dir) / self.name / "raw"
        fid, md5 = _RMD17[mol]
        d = np.load(fetch(_FIGSHARE.format(fid), root / f"rmd17_{mol}.npz", md5))
        z = d["nuclear_charges"].astype(np.int64)
        scale = 1.0 if units != "eV" else UNITS["kcal_mol_to_ev"]
        build = lambda idx: [{"pos": d["coords"][i], "atomic_numbers": z, "energy": float(d["energies"][i]) * scale,  # noqa: E731
                              "forces": d["forces"][i] * scale} for i in idx]
        if split == "all":
            return build(range(len(d["energies"])))

        def indices(part):
            if (part, int(fold)) not in _RMD17_SPLITS:
                raise ValueError(f"fold must be 1-5, got {fold!r}")
            fid2, md52 = _RMD17_SPLITS[part, int(fold)]
            path = fetch(_FIGSHARE.format(fid2), root / f"index_{part}_{int(fold):02d}.csv", md52)
            return [int(v) for v in np.loadtxt(path, dtype=np.int64).ravel()]
        tr, te = indices("train"), indices("test")
        tr, te = tr[:n_train] if n_train else tr, te[:n_test] if n_test else te
        return select_split({"train": build(tr), "test": build(te)}, split)


class QM7(DatasetBuilder):
    name = "qm7"
    description = "QM7: 7165 GDB-13 molecules, PBE0 atomization energies (5 published folds)."

    def load(self, *, split=None, cache_dir: Path, fold: int = 1, units: str = "eV", n_train: Optional[int] = None,
             n_test: Optional[int] = None):
        from scipy.io import loadmat
        if not 1 <= int(fold) <= 5:
            raise ValueError(f"fold must be 1-5, got {fold!r}")
        raw = loadmat(fetch(_QM7[0], Path(cache_dir) / self.name / "raw" / "qm7.mat", _QM7[1]))
        R, Z, T, P = raw["R"], raw["Z"], raw["T"].reshape(-1), raw["P"]
        es = UNITS["kcal_mol_to_ev"] if units == "eV" else 1.0
        rs = UNITS["bohr_to_angstrom"] if units == "eV" else 1.0

        def build(idx):
            out = []
            for i in idx:
                keep = Z[i] > 0
                out.append({"pos": np.asarray(R[i][keep], dtype=np.float64) * rs,
                            "atomic_numbers": np.asarray(Z[i][keep], dtype=np.int64), "energy": float(T[i]) * es})
            return out
        if split == "all":
            return build(range(len(T)))
        te = np.sort(P[int(fold) - 1].astype(np.int64))
        tr = np.sort(np.concatenate([P[k] for k in range(5) if k != int(fold) - 1]).astype(np.int64))
        tr, te = tr[:n_train] if n_train else tr, te[:n_test] if n_test else te
        return select_split({"train": build(tr), "test": build(te)}, split)


class ArgonMD(DatasetBuilder):
    name = "argon_md"
    description = "Periodic argon configurations with energies, forces and stress (argon_train.xyz / argon_test.xyz)."

    def load(self, *, split=None, cache_dir: Path):
        from ..io import read_extxyz
        root = Path(cache_dir) / self.name
        out = {}
        for part in ("train", "test"):
            path = root / f"argon_{part}.xyz"
            if not path.exists():
                raise FileNotFoundError(f"missing {path}")
            out[part] = [s for s in read_extxyz(str(path), energy_key="REF_energy", forces_key="REF_forces",
                                                stress_key="REF_stress")
                         if s.get("config_type") != "IsolatedAtom"]
        return select_split(out, split)


class LocalFile(DatasetBuilder):
    name = "file"
    description = "Any structure file read by xnn_b200.data.io.read_structures (extxyz, RuNNer input.data, .pt, .npz)."

    def load(self, *, split=None, cache_dir: Path, path: Optional[str] = None, **kwargs):
        from ..io import read_structures
        if path is None:
            raise ValueError("the 'file' dataset needs `path`")
        return read_structures(path, **kwargs)


class Synthetic(DatasetBuilder):
    name = "synthetic"
    description = ("Seeded synthetic benchmark sets with float64 Morse labels: 'organic' (config 2 molecules), "
                   "'small_organic' (config 1), 'crystals' (config 3), 'water' (configs 4 and 5 boxes).")

    def load(self, *, split=None, cache_dir: Path, kind: str = "organic", n: int = 64, seed: int = 0, **kwargs):
        from .. import synthetic as S
        if kind == "organic":
            items = S.organic_molecules(n, seed=seed, **kwargs)
        elif kind == "small_organic":
            items = S.small_organic(n, seed=seed, **kwargs)
        elif kind == "crystals":
            items = S.triclinic_crystals(n, seed=seed, **kwargs)
        elif kind == "water":
            items = [S.water_box(n, seed=seed, **kwargs)]
        else:
            raise ValueError(f"unknown synthetic kind {kind!r}")
        if split is None or split == "all":
            return items
        cut = int(0.9 * len(items))
        return select_split({"train": items[:cut], "test": items[cut:]}, split)


for _b in (RMD17(), QM7(), ArgonMD(), LocalFile(), Synthetic()):
    register_dataset(_b)
