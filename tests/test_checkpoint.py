"""Checkpoint compatibility: the drop-in modules expose exactly the reference's
state-dict keys, shapes and dtypes (fixture minted from the reference modules
by tests/golden/make_golden.py), so reference checkpoints load unchanged."""

import io
import json

import torch

from tests._util import GOLDEN


def _ours():
    from isa_b200.operators.cim import CIMLinear, HybridFFN, PhysicalFFN
    return {"CIMLinear": CIMLinear(12, 20), "PhysicalFFN": PhysicalFFN(12, 20), "HybridFFN": HybridFFN(12, 20)}


def test_state_dict_layout_matches_reference():
    ref = json.loads((GOLDEN / "reference_state_dict_layout.json").read_text())
    for name, mod in _ours().items():
        got = {k: [list(v.shape), str(v.dtype)] for k, v in mod.state_dict().items()}
        assert got == ref[name], name


def test_checkpoint_round_trip_and_cross_load():
    mods = _ours()
    src = mods["PhysicalFFN"]
    with torch.no_grad():
        src.fc1.vth_pos.add_(0.01)
        src.fc1.r_tia_log_scale.fill_(0.25)
    buf = io.BytesIO()
    torch.save(src.state_dict(), buf)
    buf.seek(0)
    from isa_b200.operators.cim import PhysicalFFN
    dst = PhysicalFFN(12, 20)
    dst.load_state_dict(torch.load(buf), strict=True)
    for (k, a), (_, b) in zip(src.state_dict().items(), dst.state_dict().items()):
        assert torch.equal(a, b), k
    # the measured-deployment subclass loads a plain CIMLinear checkpoint (reference operator.py:43-48)
    from isa_b200.operators.measured import DeploymentAwareCIMLinear
    layer = DeploymentAwareCIMLinear.from_cimlinear(src.fc1)
    assert torch.equal(layer.vth_pos, src.fc1.vth_pos)


def test_language_model_layout_matches_reference():
    """GPT2Model with hybrid / physical FFNs: the same state-dict keys, shapes and
    dtypes as the reference GPT2Model (fixture by
    tests/golden/make_language_layout.py), so the GPT-side wrappers (HybridFFN's
    ``cim1``, GPT2PhysicalFFN's ``cim_ffn``) load reference checkpoints."""
    from isa_b200.language import GPT2Model, ModelConfig
    ref = json.loads((GOLDEN / "reference_language_state_dict_layout.json").read_text())
    for kind in ("hybrid", "physical"):
        cfg = ModelConfig.from_preset("tiny", kind, max_seq_len=64)
        cfg.depth = 2
        got = {k: [list(v.shape), str(v.dtype)] for k, v in GPT2Model(cfg).state_dict().items()}
        assert got == ref[kind], kind
