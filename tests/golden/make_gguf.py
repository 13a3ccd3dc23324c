"""Writes small synthetic GGUF files for the GGUF-ingest tests (the GGUF v3 layout:
little-endian header, metadata key/values, tensor infos, 32-byte aligned data).

The model is a qwen35moe-shaped MoE FFN stack at test size: router f32
[ne0=d, ne1=E], experts [ne0, ne1, E] in Q8_0 or Q4_0, a shared expert and its
gate vector, values from the oracle's seeded generator and quantisers. Q4_0 can
be written in GGML's nibble order (element j low / j + 16 high nibble of byte j)
or the reference's (elements 2i, 2i + 1 in byte i).
"""
from __future__ import annotations

import struct
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1] / "oracle"))

T_U32, T_F32, T_STR, T_ARR, T_U64 = 4, 6, 8, 9, 10
GGML_F32, GGML_Q4_0, GGML_Q8_0 = 0, 2, 8


def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _kv(key, value) -> bytes:
    out = _str(key)
    if isinstance(value, str):
        return out + struct.pack("<I", T_STR) + _str(value)
    if isinstance(value, float):
        return out + struct.pack("<If", T_F32, value)
    if isinstance(value, (list, tuple)):
        body = b"".join(struct.pack("<I", int(v)) for v in value)
        return out + struct.pack("<IIQ", T_ARR, T_U32, len(value)) + body
    return out + struct.pack("<II", T_U32, int(value))


def write_gguf(path, metadata: dict, tensors: list, alignment: int = 32):
    """tensors: [(name, shape (ne0 first), ggml type, uint8 bytes)]."""
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(metadata))
    head += b"".join(_kv(k, v) for k, v in metadata.items())
    off, infos, blobs = 0, b"", []
    for name, shape, t, data in tensors:
        infos += _str(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", n) for n in shape)
        infos += struct.pack("<IQ", t, off)
        data = np.ascontiguousarray(data, np.uint8).tobytes()
        pad = (-len(data)) % alignment
        blobs.append(data + b"\0" * pad)
        off += len(data) + pad
    head += infos
    head += b"\0" * ((-len(head)) % alignment)
    Path(path).write_bytes(head + b"".join(blobs))


def q4_reference_to_ggml(raw) -> np.ndarray:
    """Inverse of the loader's GGML -> reference rewrite of Q4_0 blocks."""
    b = np.asarray(raw, np.uint8).reshape(-1, 18)
    qs = b[:, 2:]
    nib = np.empty((b.shape[0], 32), np.uint8)
    nib[:, 0::2], nib[:, 1::2] = qs & 0x0F, qs >> 4  # elements in order
    out = b.copy()
    out[:, 2:] = nib[:, :16] | (nib[:, 16:] << 4)
    return out.reshape(-1)


def moe_model(d=1024, E=8, k=2, f=256, layers=2, qtype=GGML_Q8_0, q4_order="ggml", seed=0):
    """(metadata, tensors, per-layer reference tensors) of a synthetic MoE stack."""
    import pi_oracle as orc

    meta = {"general.architecture": "qwen35moe", "general.name": "synthetic-moe-test",
            "qwen35moe.embedding_length": d, "qwen35moe.block_count": layers, "qwen35moe.expert_count": E,
            "qwen35moe.expert_used_count": k, "general.alignment": 32}
    tensors, ref = [], []
    for li in range(layers):
        s = lambda n: orc.stream_seed(seed, n, li)
        router = orc.synth_normal(s("router"), E * d, 0.02)
        mats = {n: orc.synth_quant(s(n), E, *(rc), qtype) for n, rc in
                (("gate_exps", (f, d)), ("up_exps", (f, d)), ("down_exps", (d, f)))}
        sh = {n: orc.synth_quant(s(n), 1, *(rc), qtype) for n, rc in
              (("gate_shexp", (f, d)), ("up_shexp", (f, d)), ("down_shexp", (d, f)))}
        gi = orc.synth_normal(s("gate_inp_shexp"), d, 0.02)
        ref.append(dict(router=router, **mats, shared=(sh["gate_shexp"], sh["up_shexp"], sh["down_shexp"], gi)))
        enc = (lambda a: q4_reference_to_ggml(a)) if (qtype == GGML_Q4_0 and q4_order == "ggml") else (lambda a: a)
        p = f"blk.{li}."
        tensors += [(p + "ffn_gate_inp.weight", (d, E), GGML_F32, router.view(np.uint8)),
                    (p + "ffn_gate_exps.weight", (d, f, E), qtype, enc(mats["gate_exps"])),
                    (p + "ffn_up_exps.weight", (d, f, E), qtype, enc(mats["up_exps"])),
                    (p + "ffn_down_exps.weight", (f, d, E), qtype, enc(mats["down_exps"])),
                    (p + "ffn_gate_shexp.weight", (d, f), qtype, enc(sh["gate_shexp"])),
                    (p + "ffn_up_shexp.weight", (d, f), qtype, enc(sh["up_shexp"])),
                    (p + "ffn_down_shexp.weight", (f, d), qtype, enc(sh["down_shexp"])),
                    (p + "ffn_gate_inp_shexp.weight", (d,), GGML_F32, gi.view(np.uint8))]
    return meta, tensors, ref


if __name__ == "__main__":
    out = Path(sys.argv[1] if len(sys.argv) > 1 else "synthetic_moe_q8.gguf")
    meta, tensors, _ = moe_model()
    write_gguf(out, meta, tensors)
    print(out, out.stat().st_size)
