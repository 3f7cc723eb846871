"""State-dict layout of the reference's GPT-2 models (checkpoint compatibility).

Run in a container that has the reference source tree (NOT on the GPU box):

    python tests/golden/make_language_layout.py /path/to/reference

Builds the reference ``GPT2Model`` (``src/isa/language/models.py``) at the
``tiny`` preset (two blocks) for the hybrid and physical FFN variants on the CPU and writes
every state-dict key with its shape and dtype to
``reference_language_state_dict_layout.json``.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    import torch

    from isa.language.config import ModelConfig
    from isa.language.models import GPT2Model

    torch.manual_seed(0)
    layout = {}
    for kind in ("hybrid", "physical"):
        cfg = ModelConfig.from_preset("tiny", kind, max_seq_len=64)
        cfg.depth = 2
        sd = GPT2Model(cfg).state_dict()
        layout[kind] = {k: [list(v.shape), str(v.dtype)] for k, v in sd.items()}
    (HERE / "reference_language_state_dict_layout.json").write_text(json.dumps(layout, indent=1, sort_keys=True))
    print("saved", {k: len(v) for k, v in layout.items()})


if __name__ == "__main__":
    main(sys.argv[1])
