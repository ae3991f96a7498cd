"""Loader for the golden fixtures in tests/golden/ (made by tests/golden/make_golden.py from
the reference's own Python) and the seeded inputs they were made from."""
from __future__ import annotations

import os

import numpy as np
import torch

import oracle as O
from tests.golden import make_golden as MG

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: torch.from_numpy(z[k].copy()) for k in z.files}


def bf16(t: torch.Tensor) -> torch.Tensor:
    """bf16 tensor stored as its int16 bit pattern."""
    return t.view(torch.bfloat16)


def native_inputs(mode: str):
    cfg = MG.NATIVE
    b, H, P, N, G, seed = (cfg[k] for k in ("b", "H", "P", "N", "G", "seed"))
    steps = cfg["steps"] if mode == "stale" else cfg["steps_modes"]
    xs, dts, Bs, Cs = O.make_inputs(b, H, P, G, N, steps, seed=seed, io_dtype=torch.bfloat16)
    return dict(cfg=cfg, steps=steps, xs=xs, dts=dts, Bs=Bs, Cs=Cs, s0=MG.state0(b, H, P, N, seed))


def vllm_inputs():
    cfg = MG.VLLM
    b, H, P, N, G, seed = (cfg[k] for k in ("b", "H", "P", "N", "G", "seed"))
    xs, dts, Bs, Cs = O.make_inputs(b, H, P, G, N, cfg["steps"], seed=seed, io_dtype=torch.bfloat16)
    return dict(cfg=cfg, steps=cfg["steps"], xs=xs, dts=dts, Bs=Bs, Cs=Cs,
                s0=MG.state0(b, H, P, N, seed), slots=torch.tensor(cfg["slots"]))


def check_sums(d: dict, inp: dict, prefix: str = "") -> None:
    """The regenerated inputs are the ones the fixture was made from."""
    for k, t in (("x", inp["xs"]), ("dt", inp["dts"]), ("B", inp["Bs"]), ("C", inp["Cs"]), ("s0", inp["s0"])):
        assert float(d[f"{prefix}sum_{k}"]) == MG.checksum(t), f"regenerated input {k} differs from the fixture's"


def conv_case():
    """Inputs of native_decode_conv.npz (regenerated from their seed)."""
    return MG.CONV, MG.conv_inputs(MG.CONV)
