"""Readers for the committed golden fixtures in tests/golden/ (written by make_golden.py)."""

import json
import pathlib

import numpy as np

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Raw bf16 bits (uint16) to the float32 values they encode, exactly."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {key: f[key] for key in f.files}


def manifest() -> dict:
    return json.loads((GOLDEN / "manifest.json").read_text())


def names(kind: str) -> list[str]:
    return sorted(n for n, meta in manifest().items() if meta["kind"] == kind)
