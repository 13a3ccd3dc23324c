"""Generates the committed golden fixtures for BASELINE config 1 (tiny MoE).

Inputs come from the seeded host generator (SplitMix64 + Box-Muller,
libpi_moe.so's pi_synth_normal_host) and the oracle's Q8_0 weight quantiser;
outputs come from the CPU oracle (oracle/pi_oracle.cpp, the restatement of
the reference's CPU path). The reference itself (Rust) cannot be built in
this image, so these fixtures pin the oracle against regressions; the
reference's own known-answer tests are in reference_kat.json.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

import pi_oracle as orc  # noqa: E402
from powerinfer_x64_b200 import synth  # noqa: E402


def c1_inputs(seed: int = 0):
    c = synth.C1
    s = lambda n: synth.stream_seed(seed, n)
    router = synth.normal_host(s("router"), c.E * c.d, 0.02)
    g = orc.quantize_q8_0(synth.normal_host(s("gate_exps"), c.E * c.f * c.d, 0.02))
    u = orc.quantize_q8_0(synth.normal_host(s("up_exps"), c.E * c.f * c.d, 0.02))
    dn = orc.quantize_q8_0(synth.normal_host(s("down_exps"), c.E * c.d * c.f, 0.02))
    x = synth.normal_host(s("x"), c.T[0] * c.d, 1.0).reshape(c.T[0], c.d)
    return dict(router=router, gate_exps=g, up_exps=u, down_exps=dn, x=x)


def digest(inp) -> str:
    h = hashlib.sha256()
    for k in sorted(inp):
        h.update(k.encode())
        h.update(np.ascontiguousarray(inp[k]).tobytes())
    return h.hexdigest()


def main():
    c = synth.C1
    inp = c1_inputs(0)
    r = orc.moe_route(inp["x"], inp["router"], c.d, c.E, c.k)
    out = orc.moe_layer(inp["x"], c.d, c.f, c.E, c.k, c.qtype, inp["router"], inp["gate_exps"], inp["up_exps"],
                        inp["down_exps"], threads=1)
    path = Path(__file__).resolve().parent / "c1_seed0.npz"
    np.savez_compressed(path, input_sha256=np.array(digest(inp)), idx=r["idx"], gates=r["gates"],
                        counts=r["counts"], offsets=r["offsets"], perm=r["perm"], logits=r["logits"], out=out)
    print(path, digest(inp))


if __name__ == "__main__":
    main()
