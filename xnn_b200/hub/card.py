"""Model cards of portable model directories (``card.json``)."""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional, Union

CARD_FILE = "card.json"
CONFIG_FILE = "config.yaml"
WEIGHTS_FILE = "model.pt"


@dataclass
class ModelCard:
    """What a portable model directory holds (name, model family, species, cutoff, license...)."""

    name: str = ""
    model: str = ""
    description: str = ""
    license: str = ""
    species: List[int] = field(default_factory=list)
    cutoff: Optional[float] = None
    dtype: str = "float32"
    heads: List[str] = field(default_factory=list)
    md5: str = ""
    extra: Dict[str, Any] = field(default_factory=dict)

    def write(self, path: Union[str, Path]) -> Path:
        p = Path(path)
        p.write_text(json.dumps(asdict(self), indent=2, sort_keys=True) + "\n")
        return p

    @classmethod
    def read(cls, path: Union[str, Path]) -> "ModelCard":
        d = json.loads(Path(path).read_text())
        known = {k: d.pop(k) for k in list(d) if k in cls.__dataclass_fields__}
        card = cls(**known)
        card.extra.update(d)
        return card
