"""Small seeded routed-MoE cases shared by the CPU and GPU tests."""
from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "gyro-dx_b200"))

from gyro_moe import synth  # noqa: E402


def small_layer(seed: int = 11, type_id: int = 144, n_tok: int = 5):
    """E=256, F=128, 16 experts, top-4, with signs; n_tok f32 tokens."""
    layer = synth.make_layer(seed, n_expert=16, E=256, F=128, U=4, type_id=type_id)
    x = synth.tokens(seed + 1000, n_tok, E=256)
    return layer, x
