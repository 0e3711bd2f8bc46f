"""Real-weight loading: MLX safetensors checkpoints and RNLMOE01 layer datasets.

Three pieces, following the reference's tooling:

* :class:`TensorStore` indexes every ``*.safetensors`` file of a checkpoint
  directory by tensor name and reads single tensors (with the SHA-256 of their
  raw bytes), like ``SafeTensorStore`` in bench/export_ornith_moe_layer.py:25-61.
  :func:`write_safetensors` writes the same container (tests, tools).
* :func:`export_layer` derives one layer's two-stage probe dataset -- the
  RNLMOE01 binary of bench/export_ornith_moe_layer.py:86-183: the routed
  experts with up||gate packed on axis 1, a seeded activation row and eight
  seeded router weights -- plus its manifest of tensor hashes.
  :func:`read_layer_dataset` parses it back with the checks of the native
  probe's loader (native/src/fused_moe_probe.mm:539-590).
* :func:`load_block` builds a whole :class:`runnel_b200.ops.BlockTensors`
  (router, routed experts, shared expert and its gate) from a checkpoint
  layer, by the mlx-lm Qwen3.5 MoE names.  Real checkpoints quantize the
  router and the shared-expert gate to 8 bits (80 per-tensor overrides,
  reference tests/test_checkpoint.py:149-152); the block takes them as they
  are stored (router_bits 8: codes, scales and biases), and the arrays also
  carry a bf16 dequantisation (s*q + b in fp32, rounded) for plain-torch use.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

from .quant import f32_to_bf16_bits, bf16_bits_to_f32, unpack_codes

MAGIC = b"RNLMOE01"
_HEADER = struct.Struct("<8s8I")  # magic, version, bits, total, selected, gate/up rows, down rows, H, I
_DTYPES = {"U32": "<u4", "BF16": "<u2", "F32": "<f4", "F16": "<f2", "U8": "u1", "I32": "<i4", "U16": "<u2"}
_DATASET_SEED = 0x4F524E495448  # "ORNITH": the exporter's activation / router-weight generator


def _sha256(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


class TensorStore:
    """Name -> (file, byte range, shape, dtype) over a checkpoint directory."""

    def __init__(self, root: str):
        self.root = root
        self.entries: dict[str, tuple[str, tuple[int, int], tuple[int, ...], str]] = {}
        names = sorted(n for n in os.listdir(root) if n.endswith(".safetensors"))
        if not names:
            raise FileNotFoundError(f"no .safetensors files in {root}")
        for n in names:
            path = os.path.join(root, n)
            with open(path, "rb") as f:
                size = struct.unpack("<Q", f.read(8))[0]
                header = json.loads(f.read(size))
            for name, meta in header.items():
                if name == "__metadata__":
                    continue
                self.entries[name] = (path, tuple(meta["data_offsets"]), tuple(meta["shape"]), meta["dtype"])

    def __contains__(self, name: str) -> bool:
        return name in self.entries

    def read(self, name: str) -> tuple[np.ndarray, str]:
        """(array, sha256 of its raw bytes); KeyError names a missing tensor."""
        if name not in self.entries:
            raise KeyError(f"tensor is missing: {name}")
        path, (a, b), shape, dtype = self.entries[name]
        if dtype not in _DTYPES:
            raise ValueError(f"unsupported tensor dtype {dtype} for {name}")
        with open(path, "rb") as f:
            size = struct.unpack("<Q", f.read(8))[0]
            f.seek(8 + size + a)
            raw = f.read(b - a)
        if len(raw) != b - a:
            raise ValueError(f"{path} is truncated at {name}")
        return np.frombuffer(raw, dtype=_DTYPES[dtype]).copy().reshape(shape), _sha256(raw)


def write_safetensors(path: str, tensors: dict[str, tuple[np.ndarray, str]], metadata: dict | None = None) -> None:
    """Write {name: (array, safetensors dtype)} as one safetensors file."""
    header, blobs, off = {}, [], 0
    for name, (arr, dtype) in tensors.items():
        raw = np.ascontiguousarray(arr, dtype=_DTYPES[dtype]).tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for raw in blobs:
            f.write(raw)


# ------------------------------------------------------------ layer names

def layer_prefix(layer: int) -> str:
    return f"language_model.model.layers.{layer}.mlp"


def _routed_names(layer: int) -> dict[str, str]:
    p = f"{layer_prefix(layer)}.switch_mlp"
    return {f"{proj}_{part}": f"{p}.{proj}_proj.{part}" for proj in ("gate", "up", "down")
            for part in ("weight", "scales", "biases")}


def _bits_of(packed_width: int, K: int) -> int:
    for bits in (4, 8):
        if packed_width == K * bits // 32:
            return bits
    return 0


def read_routed(store: TensorStore, layer: int) -> tuple[dict, dict]:
    """The routed bank of one layer, packed: (arrays, tensor hashes).

    Arrays: gu_w [E, 2I, H*b/32] (up rows then gate rows), gu_s, gu_b, dn_w,
    dn_s, dn_b and ``bits``.  Shape checks and messages follow
    bench/export_ornith_moe_layer.py:108-124."""
    t, hashes = {}, {}
    for label, name in _routed_names(layer).items():
        t[label], hashes[name] = store.read(name)
    g, u, d = t["gate_weight"], t["up_weight"], t["down_weight"]
    if g.ndim != 3 or u.shape != g.shape:
        raise ValueError("gate/up tensor shapes do not agree")
    if d.ndim != 3:
        raise ValueError("down tensor is not an expert matrix")
    E, I, gp = g.shape
    if d.shape[0] != E or d.shape[1] != I * 4:
        raise ValueError("down tensor shape is inconsistent with gate/up rows")
    H = d.shape[1]
    bits = _bits_of(gp, H)
    if bits == 0:
        raise ValueError(f"cannot infer quantization bits from packed width {gp}")
    if d.shape[2] != I * bits // 32:
        raise ValueError("down packed width is inconsistent with the selected bits")
    out = {
        "bits": bits,
        "gu_w": np.concatenate((u, g), axis=1), "gu_s": np.concatenate((t["up_scales"], t["gate_scales"]), axis=1),
        "gu_b": np.concatenate((t["up_biases"], t["gate_biases"]), axis=1),
        "dn_w": d, "dn_s": t["down_scales"], "dn_b": t["down_biases"],
    }
    return out, hashes


# ------------------------------------------------------ RNLMOE01 datasets

@dataclass
class LayerDataset:
    """One layer's two-stage probe dataset (RNLMOE01)."""

    bits: int
    selected: np.ndarray  # [k] u32
    gu_w: np.ndarray
    gu_s: np.ndarray
    gu_b: np.ndarray
    dn_w: np.ndarray
    dn_s: np.ndarray
    dn_b: np.ndarray
    x: np.ndarray  # [H] u16 (bf16 bits)
    route_w: np.ndarray  # [k] f32, sums to 1
    meta: dict = field(default_factory=dict)

    @property
    def E(self) -> int:
        return self.gu_w.shape[0]


def dataset_inputs(k: int = 8, H: int = 2048) -> tuple[np.ndarray, np.ndarray]:
    """The exporter's seeded activation row (U(-1,1) rounded to bf16) and k
    router weights (U(0.5,1.5), normalised in fp32)."""
    rng = np.random.default_rng(_DATASET_SEED)
    x = f32_to_bf16_bits(rng.uniform(-1.0, 1.0, size=H).astype(np.float32))
    w = rng.uniform(0.5, 1.5, size=k).astype(np.float32)
    w /= np.sum(w, dtype=np.float32)
    return x.astype(np.uint16), w


def write_layer_dataset(path: str, ds: LayerDataset) -> bytes:
    """Write RNLMOE01; returns the bytes written."""
    E, I2 = ds.gu_w.shape[0], ds.gu_w.shape[1]
    H = ds.dn_w.shape[1]
    parts = [_HEADER.pack(MAGIC, 1, ds.bits, E, len(ds.selected), I2, H, H, I2 // 2),
             np.asarray(ds.selected, "<u4").tobytes()]
    for arr, dt in ((ds.gu_w, "<u4"), (ds.gu_s, "<u2"), (ds.gu_b, "<u2"), (ds.dn_w, "<u4"), (ds.dn_s, "<u2"),
                    (ds.dn_b, "<u2"), (ds.x, "<u2"), (ds.route_w, "<f4")):
        parts.append(np.ascontiguousarray(arr, dtype=dt).tobytes())
    data = b"".join(parts)
    with open(path, "wb") as f:
        f.write(data)
    return data


def read_layer_dataset(path: str, bits: int | None = None, total_experts: int | None = None) -> LayerDataset:
    """Parse RNLMOE01 with the native loader's checks: magic and version, the
    requested bits and bank size, and no truncation."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < _HEADER.size:
        raise ValueError(f"fused MoE dataset is truncated: {path}")
    magic, version, b, E, k, I2, Hd, H, I = _HEADER.unpack_from(data)
    if magic != MAGIC or version != 1 or (bits is not None and b != bits) or \
            (total_experts is not None and E != total_experts) or I2 != 2 * I or Hd != H or b not in (4, 8):
        raise ValueError("fused MoE dataset header does not match the requested probe")
    off = _HEADER.size
    shapes = [("selected", (k,), "<u4"), ("gu_w", (E, I2, H * b // 32), "<u4"), ("gu_s", (E, I2, H // 64), "<u2"),
              ("gu_b", (E, I2, H // 64), "<u2"), ("dn_w", (E, H, I * b // 32), "<u4"),
              ("dn_s", (E, H, I // 64), "<u2"), ("dn_b", (E, H, I // 64), "<u2"), ("x", (H,), "<u2"),
              ("route_w", (k,), "<f4")]
    out = {}
    for name, shape, dt in shapes:
        n = int(np.prod(shape)) * np.dtype(dt).itemsize
        if off + n > len(data):
            raise ValueError(f"fused MoE dataset is truncated: {path}")
        out[name] = np.frombuffer(data, dtype=dt, count=int(np.prod(shape)), offset=off).reshape(shape).copy()
        off += n
    if np.any(out["selected"] >= E):
        raise ValueError("fused MoE dataset expert selection is outside the bank")
    return LayerDataset(bits=b, meta={"sha256": _sha256(data), "bytes": len(data)}, **out)


def export_layer(store: TensorStore, layer: int, selected, output: str, manifest: str | None = None,
                 model_name: str | None = None) -> dict:
    """Write one layer's RNLMOE01 dataset and its manifest; returns the manifest."""
    sel = [int(e) for e in selected]
    if len(sel) != 8 or len(set(sel)) != 8 or any(e < 0 for e in sel):
        raise ValueError("--experts must contain eight unique non-negative indices")
    routed, hashes = read_routed(store, layer)
    E = routed["gu_w"].shape[0]
    if any(e >= E for e in sel):
        raise ValueError("selected expert is outside the checkpoint")
    x, rw = dataset_inputs(8, routed["dn_w"].shape[1])
    ds = LayerDataset(bits=routed["bits"], selected=np.asarray(sel, np.uint32), x=x, route_w=rw,
                      **{k: routed[k] for k in ("gu_w", "gu_s", "gu_b", "dn_w", "dn_s", "dn_b")})
    data = write_layer_dataset(output, ds)
    man = {"schema_version": 1, "model_name": model_name or os.path.basename(os.path.normpath(store.root)),
           "layer": layer, "bits": ds.bits, "total_experts": E, "selected_experts": sel,
           "gate_up_shape": list(ds.gu_w.shape), "down_shape": list(ds.dn_w.shape), "tensor_sha256": hashes,
           "output_sha256": _sha256(data), "output_bytes": len(data),
           "note": "temporary derived artifact; model weights are not committed"}
    mpath = manifest or os.path.splitext(output)[0] + ".manifest.json"
    with open(mpath, "w") as f:
        f.write(json.dumps(man, indent=2, sort_keys=True) + "\n")
    return man


# ------------------------------------------------------------ whole block

def _dequant_bf16(w: np.ndarray, s: np.ndarray, b: np.ndarray, bits: int) -> np.ndarray:
    q = unpack_codes(w, bits).astype(np.float32)
    sf = np.repeat(bf16_bits_to_f32(s), 64, axis=-1)
    bf = np.repeat(bf16_bits_to_f32(b), 64, axis=-1)
    return f32_to_bf16_bits((sf * q + bf).astype(np.float32)).astype(np.uint16)


def _dense_bf16(store: TensorStore, base: str, K: int) -> np.ndarray:
    """A Linear's weight as bf16 bits: stored bf16, or 8/4-bit affine dequantised."""
    w, _ = store.read(f"{base}.weight")
    if w.dtype == np.uint16:
        return w
    s, _ = store.read(f"{base}.scales")
    b, _ = store.read(f"{base}.biases")
    bits = _bits_of(w.shape[-1], K)
    if bits == 0:
        raise ValueError(f"cannot infer quantization bits of {base}")
    return _dequant_bf16(w, s, b, bits)


def _affine8(store: TensorStore, base: str, K: int):
    """(codes, scales, biases) of an 8-bit affine Linear, else None."""
    w, _ = store.read(f"{base}.weight")
    if w.dtype != np.uint32 or _bits_of(w.shape[-1], K) != 8:
        return None
    return w, store.read(f"{base}.scales")[0], store.read(f"{base}.biases")[0]


def load_block_arrays(store: TensorStore, layer: int) -> dict:
    """numpy arrays of a layer's whole MoE block (fields of SyntheticBlock).

    An 8-bit router and shared gate come as stored (router_bits 8, router_q /
    router_s / router_b, sgate_q / sgate_s / sgate_b) and, in router_w /
    shared_gate_w, as their bf16 dequantisation."""
    routed, _ = read_routed(store, layer)
    bits = routed["bits"]
    H = routed["dn_w"].shape[1]
    p = layer_prefix(layer)
    out = dict(routed)
    out["router_w"] = _dense_bf16(store, f"{p}.gate", H)
    out["router_bits"] = 16
    q8 = _affine8(store, f"{p}.gate", H)
    if q8 is not None:
        out["router_bits"] = 8
        out["router_q"], out["router_s"], out["router_b"] = q8
    sh = f"{p}.shared_expert"
    if f"{sh}.up_proj.weight" in store:
        parts = {}
        for proj in ("gate", "up", "down"):
            for part in ("weight", "scales", "biases"):
                parts[(proj, part)] = store.read(f"{sh}.{proj}_proj.{part}")[0]
        if _bits_of(parts[("up", "weight")].shape[-1], H) != bits:
            raise ValueError("shared expert bits differ from the routed experts'")
        # packed on axis 0 like the routed pair: up rows, then gate rows
        out["sgu_w"] = np.concatenate((parts[("up", "weight")], parts[("gate", "weight")]), axis=0)
        out["sgu_s"] = np.concatenate((parts[("up", "scales")], parts[("gate", "scales")]), axis=0)
        out["sgu_b"] = np.concatenate((parts[("up", "biases")], parts[("gate", "biases")]), axis=0)
        out["sdn_w"], out["sdn_s"], out["sdn_b"] = (parts[("down", p2)] for p2 in ("weight", "scales", "biases"))
        out["shared_gate_w"] = _dense_bf16(store, f"{p}.shared_expert_gate", H).reshape(-1)
        g8 = _affine8(store, f"{p}.shared_expert_gate", H)
        if (g8 is not None) != (q8 is not None):
            raise ValueError("the router and the shared-expert gate must both be 8-bit, or both not")
        if g8 is not None:
            out["sgate_q"], out["sgate_s"], out["sgate_b"] = (v.reshape(-1) for v in g8)
    norm = f"language_model.model.layers.{layer}.post_attention_layernorm.weight"
    if norm in store:
        out["norm_w"] = store.read(norm)[0]
    return out


def load_block(store: TensorStore, layer: int, device="cuda", E_range: tuple[int, int] | None = None):
    """A layer's whole block as :class:`runnel_b200.ops.BlockTensors`."""
    import torch

    from .ops import BlockTensors

    a = load_block_arrays(store, layer)
    lo, hi = E_range if E_range else (0, a["gu_w"].shape[0])

    def up(arr, bf16=False):
        t = torch.from_numpy(np.ascontiguousarray(arr).view(np.int32 if arr.dtype == np.uint32 else np.int16))
        t = t.view(torch.uint32) if arr.dtype == np.uint32 else (t.view(torch.bfloat16) if bf16 else t)
        return t.to(device)

    q8 = a["router_bits"] == 8
    bt = BlockTensors(bits=a["bits"], gu_w=up(a["gu_w"][lo:hi]), gu_s=up(a["gu_s"][lo:hi], True),
                      gu_b=up(a["gu_b"][lo:hi], True), dn_w=up(a["dn_w"][lo:hi]), dn_s=up(a["dn_s"][lo:hi], True),
                      dn_b=up(a["dn_b"][lo:hi], True),
                      router_w=up(a["router_q"]) if q8 else up(a["router_w"], True),
                      E_total=a["gu_w"].shape[0], expert_offset=lo)
    if q8:
        bt.router_bits = 8
        bt.router_s, bt.router_b = up(a["router_s"], True), up(a["router_b"], True)
    if "sgu_w" in a:
        if q8:
            bt.shared_gate_w = up(a["sgate_q"])
            bt.sgate_s, bt.sgate_b = up(a["sgate_s"], True), up(a["sgate_b"], True)
        else:
            bt.shared_gate_w = up(a["shared_gate_w"], True)
        bt.sgu_w, bt.sdn_w = up(a["sgu_w"]), up(a["sdn_w"])
        bt.sgu_s, bt.sgu_b = up(a["sgu_s"], True), up(a["sgu_b"], True)
        bt.sdn_s, bt.sdn_b = up(a["sdn_s"], True), up(a["sdn_b"], True)
    return bt
