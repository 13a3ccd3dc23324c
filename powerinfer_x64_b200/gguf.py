"""GGUF ingest for the MoE path: the reader of the reference's ``GgufFile``
(src/gguf/mod.rs:17-181) and ``WeightTensor`` windows (src/weights.rs:20-113),
restated from the GGUF v2/v3 file layout (the reference parses it with the
``gguf-rs`` crate): a little-endian header, metadata key/values, tensor infos,
then the tensor data at ``general.alignment`` (default 32).

Tensors are zero-copy windows into a read-only memory map, like the reference's
``Arc<Mmap>``. ``moe_layer`` builds a device ``MoeLayer`` (or an ``EPMoeLayer``
holding one rank's experts) straight from a layer's ``blk.N.ffn_*`` tensors.

Q4_0 nibble order: GGML stores element j of a block in the low nibble of byte
j and element j + 16 in the high nibble; the reference decodes byte i as
elements 2i (low) and 2i + 1 (high) (quant/mod.rs:193-199), and the kernels
here follow the reference. ``q4_order="ggml"`` rewrites Q4_0 blocks of a real
GGML file into the reference's order at load, so the layer computes what the
file means; ``"reference"`` (default) keeps the bytes, i.e. the reference's
own reading of the file.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

GGUF_MAGIC = b"GGUF"
# GGUF metadata value types
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f", T_BOOL: "<?",
           T_U64: "<Q", T_I64: "<q", T_F64: "<d"}
# ggml tensor types this path reads: (block elements, block bytes)
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8
BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q4_0: (32, 18), GGML_Q8_0: (32, 34)}


class GgufError(ValueError):
    pass


@dataclass
class TensorInfo:
    name: str
    shape: tuple  # (ne0, ne1, ...), ne0 fastest
    ggml_type: int
    offset: int   # from the start of the data section
    nbytes: int


class _Reader:
    def __init__(self, buf):
        self.b, self.p = buf, 0

    def take(self, fmt):
        v = struct.unpack_from(fmt, self.b, self.p)[0]
        self.p += struct.calcsize(fmt)
        return v

    def string(self):
        n = self.take("<Q")
        s = bytes(self.b[self.p:self.p + n])
        self.p += n
        return s.decode("utf-8")

    def value(self, t):
        if t in _SCALAR:
            return self.take(_SCALAR[t])
        if t == T_STR:
            return self.string()
        if t == T_ARR:
            et, n = self.take("<I"), self.take("<Q")
            return [self.value(et) for _ in range(n)]
        raise GgufError(f"unknown metadata value type {t}")


def tensor_nbytes(shape, ggml_type) -> int:
    if ggml_type not in BLOCK:
        raise GgufError(f"tensor type {ggml_type} is not read by this path")
    n = int(np.prod(shape)) if len(shape) else 1
    ve, be = BLOCK[ggml_type]
    return -(-n // ve) * be


class GgufFile:
    """A GGUF file opened read-only (src/gguf/mod.rs:17-34)."""

    def __init__(self, path):
        self.path = Path(path)
        self._f = open(self.path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        r = _Reader(self._mm)
        if bytes(self._mm[:4]) != GGUF_MAGIC:
            raise GgufError(f"{path}: not a GGUF file")
        r.p = 4
        self.version = r.take("<I")
        if self.version not in (2, 3):
            raise GgufError(f"{path}: GGUF version {self.version} (2 or 3 expected)")
        n_tensors, n_kv = r.take("<Q"), r.take("<Q")
        self.metadata = {}
        for _ in range(n_kv):
            key = r.string()
            self.metadata[key] = r.value(r.take("<I"))
        self.tensors = {}
        for _ in range(n_tensors):
            name = r.string()
            nd = r.take("<I")
            shape = tuple(r.take("<Q") for _ in range(nd))
            t, off = r.take("<I"), r.take("<Q")
            self.tensors[name] = TensorInfo(name, shape, t, off, tensor_nbytes(shape, t))
        align = int(self.metadata.get("general.alignment", 32))
        self.data_start = -(-r.p // align) * align
        for ti in self.tensors.values():
            if self.data_start + ti.offset + ti.nbytes > len(self._mm):
                raise GgufError(f"{path}: tensor {ti.name} runs past the end of the file")

    def close(self):
        """Closes the file; the map itself goes when the last tensor view is dropped."""
        try:
            self._mm.close()
        except BufferError:  # tensor windows still reference the map
            pass
        self._f.close()

    # -- metadata (src/gguf/mod.rs:36-181) ------------------------------------
    def architecture(self) -> str:
        a = self.metadata.get("general.architecture")
        if not isinstance(a, str):
            raise GgufError("Architecture not found in GGUF metadata")
        return a

    def get_config(self, suffix: str):
        """``{arch}.{suffix}``, else ``llama.{suffix}`` (src/gguf/mod.rs:42-48)."""
        v = self.metadata.get(f"{self.architecture()}.{suffix}")
        return v if v is not None else self.metadata.get(f"llama.{suffix}")

    def embedding_length(self) -> int:
        v = self.get_config("embedding_length")
        if v is None:
            raise GgufError("Embedding length not found")
        return int(v)

    def block_count(self) -> int:
        v = self.get_config("block_count")
        if v is None:
            raise GgufError("Block count not found")
        return int(v)

    def moe_config(self):
        """(expert_count, expert_used_count, expert_intermediate_size) or None; the
        width falls back to ne1 of a ``ffn_gate_exps.weight`` (src/gguf/mod.rs:150-181)."""
        ec, eu = self.get_config("expert_count"), self.get_config("expert_used_count")
        if ec is None or eu is None:
            return None
        f = self.get_config("expert_feed_forward_length")
        if f is None:
            for ti in self.tensors.values():
                if "ffn_gate_exps.weight" in ti.name and len(ti.shape) >= 2:
                    f = ti.shape[1]
                    break
        if f is None:
            return None
        return int(ec), int(eu), int(f)

    # -- tensor windows (src/weights.rs:20-113) -------------------------------
    def raw(self, name: str) -> np.ndarray:
        """Zero-copy uint8 view of a tensor's bytes."""
        ti = self.tensor(name)
        return np.frombuffer(self._mm, np.uint8, ti.nbytes, self.data_start + ti.offset)

    def tensor(self, name: str) -> TensorInfo:
        ti = self.tensors.get(name)
        if ti is None:
            raise GgufError(f"tensor {name} not in {self.path.name}")
        return ti

    def expert_raw_slice(self, name: str, expert: int) -> np.ndarray:
        """Expert `expert`'s bytes of a [ne0, ne1, n_experts] tensor (weights.rs:78-113)."""
        ti = self.tensor(name)
        if len(ti.shape) < 3:
            raise GgufError(f"expert_raw_slice requires 3D tensor, got {len(ti.shape)}D for {name}")
        ne0, ne1, ne = ti.shape[:3]
        if expert >= ne:
            raise GgufError(f"expert_idx {expert} >= n_experts {ne} for {name}")
        per = tensor_nbytes((ne0, ne1), ti.ggml_type)
        return self.raw(name)[expert * per:(expert + 1) * per]


def q4_0_ggml_to_reference(raw) -> np.ndarray:
    """Q4_0 blocks with GGML's nibble order (element j in the low nibble of byte j,
    j + 16 in its high nibble) rewritten in the reference's order (elements 2i,
    2i + 1 in byte i). Scales are kept."""
    b = np.asarray(raw, np.uint8).reshape(-1, 18)
    qs = b[:, 2:]
    nib = np.concatenate([qs & 0x0F, qs >> 4], axis=1)  # elements 0..31 in GGML order
    out = b.copy()
    out[:, 2:] = nib[:, 0::2] | (nib[:, 1::2] << 4)
    return out.reshape(-1)


def _weights(gf: GgufFile, name: str, q4_order: str, experts=None):
    ti = gf.tensor(name)
    if experts is None:
        raw = gf.raw(name)
    else:
        lo, hi = experts
        raw = np.concatenate([gf.expert_raw_slice(name, e) for e in range(lo, hi)]) if hi - lo > 1 else \
            gf.expert_raw_slice(name, lo)
    if ti.ggml_type == GGML_Q4_0 and q4_order == "ggml":
        raw = q4_0_ggml_to_reference(raw)
    return ti, np.ascontiguousarray(raw)


def moe_layer(gf: GgufFile, layer: int, q4_order: str = "reference", rank: int = 0, world: int = 1, comm=None,
              device: int | None = None):
    """The MoE FFN of block `layer` as a device layer.

    Reads ``blk.{layer}.ffn_gate_inp.weight`` (f32 router [ne0=d, ne1=E]),
    ``ffn_{gate,up,down}_exps.weight`` (Q8_0 or Q4_0 [ne0, ne1, E]) and, when
    present, ``ffn_{gate,up,down}_shexp.weight`` with ``ffn_gate_inp_shexp.weight``
    (the tensors model/mod.rs:1245-1571 uses). world > 1 returns the EPMoeLayer
    holding rank's E/world experts (Q8_0 only).
    """
    from .moe import MoeLayer

    if q4_order not in ("reference", "ggml"):
        raise GgufError("q4_order must be 'reference' or 'ggml'")
    cfg = gf.moe_config()
    if cfg is None:
        raise GgufError("no MoE configuration (expert_count / expert_used_count) in the metadata")
    E, k, f = cfg
    d = gf.embedding_length()
    p = f"blk.{layer}."
    rt = gf.tensor(p + "ffn_gate_inp.weight")
    if rt.ggml_type != GGML_F32 or rt.shape[:2] != (d, E):
        raise GgufError(f"{p}ffn_gate_inp.weight: f32 [{d}, {E}] expected, got type {rt.ggml_type} {rt.shape}")
    router = np.frombuffer(gf.raw(p + "ffn_gate_inp.weight"), np.float32).copy()
    experts = None
    if world > 1:
        if gf.tensor(p + "ffn_gate_exps.weight").ggml_type != GGML_Q8_0:
            raise GgufError("the expert-parallel layer takes Q8_0 experts")
        if E % world:
            raise GgufError("expert_count must be a multiple of the world size")
        P = E // world
        experts = (rank * P, (rank + 1) * P)
    gt, g = _weights(gf, p + "ffn_gate_exps.weight", q4_order, experts)
    ut, u = _weights(gf, p + "ffn_up_exps.weight", q4_order, experts)
    dt, dn = _weights(gf, p + "ffn_down_exps.weight", q4_order, experts)
    qt = gt.ggml_type
    if not (qt == ut.ggml_type == dt.ggml_type) or qt not in (GGML_Q8_0, GGML_Q4_0):
        raise GgufError("expert tensors must share one type, Q8_0 or Q4_0")
    if gt.shape[:3] != (d, f, E) or ut.shape[:3] != (d, f, E) or dt.shape[:3] != (f, d, E):
        raise GgufError(f"expert tensor shapes {gt.shape} {ut.shape} {dt.shape} do not match d={d} f={f} E={E}")
    shared = None
    if p + "ffn_gate_shexp.weight" in gf.tensors:
        sg = _weights(gf, p + "ffn_gate_shexp.weight", q4_order)[1]
        su = _weights(gf, p + "ffn_up_shexp.weight", q4_order)[1]
        sd = _weights(gf, p + "ffn_down_shexp.weight", q4_order)[1]
        gi = None
        if p + "ffn_gate_inp_shexp.weight" in gf.tensors:
            gi = np.frombuffer(gf.raw(p + "ffn_gate_inp_shexp.weight"), np.float32).copy()
        shared = (sg, su, sd, gi)
    if world > 1:
        from .ep import EPMoeLayer

        return EPMoeLayer(router, g, u, dn, d, f, E, k, rank=rank, world=world, shared=shared, comm=comm,
                          device=device)
    return MoeLayer(router, g, u, dn, qt, d, f, E, k, shared=shared, device=device)
