"""Real-weight ingest: a q4f16 ONNX export of Qwen3 -> the runtime directory layout.

Restates `scripts/extract-qwen-runtime-assets.mjs` (reference): the same output files,
file names and manifest schema, read from the same initializers:

    shared/embed_tokens.f16, cos_cache.f16, sin_cache.f16, final_norm.f16   raw f16 (:27-34)
    layers/<i>/norm_{input,q,k,postAttention}.f16                           raw f16 (:44-53)
    layers/<i>/<proj>_weight_q4.bin    MatMulNBits weight [N][K/32][16] raw bytes (:74-79)
    layers/<i>/<proj>_scales_f32.bin   the f16 block scales widened to f32 (:80, :133-143)
    manifest.json                                                          (:14-25, :70)

The ONNX file is read with a small protobuf wire-format reader (ModelProto.graph ->
GraphProto.initializer -> TensorProto name / dims / data_type / raw_data), so no
`onnx` package is needed. Initializers stored as external data (data_location =
EXTERNAL, location / offset / length) are read from the file beside the model.

Where the reference hard-codes the Qwen3-0.6B dimensions (:14-25), they are derived
here from the tensors themselves (the same numbers for that model), so smaller
exports of the same architecture extract too.

    python -m kernel_optimization_webgpu_b200.onnx_ingest model_q4f16.onnx out_dir [layers]
"""
from __future__ import annotations

import json
import os
import sys
from typing import Dict, Optional, Tuple

import numpy as np

FLOAT16 = 10   # TensorProto.DataType
UINT8 = 2

PROJECTIONS = (
    ("q", "attn.q_proj.MatMul"), ("k", "attn.k_proj.MatMul"), ("v", "attn.v_proj.MatMul"),
    ("o", "attn.o_proj.MatMul"), ("gate", "mlp.gate_proj.MatMul"), ("up", "mlp.up_proj.MatMul"),
    ("down", "mlp.down_proj.MatMul"),
)
NORMS = (
    ("input", "input_layernorm.weight"), ("q", "attn.q_norm.layernorm.weight"),
    ("k", "attn.k_norm.layernorm.weight"), ("postAttention", "post_attention_layernorm.weight"),
)


# ---- protobuf wire format -----------------------------------------------------------

def _varint(buf: memoryview, i: int) -> Tuple[int, int]:
    shift = result = 0
    while True:
        b = buf[i]
        i += 1
        result |= (b & 0x7F) << shift
        if b < 0x80:
            return result, i
        shift += 7
        if shift > 63:
            raise ValueError("malformed protobuf varint")


def _fields(buf: memoryview):
    """Yield (field number, wire type, value) of one message: ints for varint and
    fixed fields, memoryviews for length-delimited ones."""
    i, n = 0, len(buf)
    while i < n:
        key, i = _varint(buf, i)
        field, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(buf, i)
        elif wt == 1:
            v = int.from_bytes(buf[i:i + 8], "little")
            i += 8
        elif wt == 2:
            ln, i = _varint(buf, i)
            if i + ln > n:
                raise ValueError("truncated protobuf message")
            v = buf[i:i + ln]
            i += ln
        elif wt == 5:
            v = int.from_bytes(buf[i:i + 4], "little")
            i += 4
        else:
            raise ValueError(f"unsupported protobuf wire type {wt}")
        yield field, wt, v


class Tensor:
    """One initializer: name, dims, ONNX data type and its raw little-endian bytes."""

    def __init__(self, name: str, dims: list, data_type: int, raw: memoryview):
        self.name, self.dims, self.data_type, self.raw = name, dims, data_type, raw

    @property
    def nbytes(self) -> int:
        return len(self.raw)


def _tensor(msg: memoryview, model_dir: str) -> Tensor:
    name, dims, dtype, raw = "", [], 0, None
    external: Dict[str, str] = {}
    location = 0
    for field, wt, v in _fields(msg):
        if field == 1:                       # dims (packed or one per field)
            if wt == 2:
                j = 0
                while j < len(v):
                    d, j = _varint(v, j)
                    dims.append(d)
            else:
                dims.append(v)
        elif field == 2:
            dtype = v
        elif field == 8:
            name = bytes(v).decode()
        elif field == 9:
            raw = v
        elif field == 13:                    # external_data: StringStringEntryProto
            kv = {f: bytes(x).decode() for f, _, x in _fields(v)}
            external[kv.get(1, "")] = kv.get(2, "")
        elif field == 14:
            location = v
    if location == 1:                        # DataLocation.EXTERNAL
        path = os.path.join(model_dir, external["location"])
        offset = int(external.get("offset", 0))
        with open(path, "rb") as f:
            f.seek(offset)
            length = int(external["length"]) if "length" in external else -1
            raw = memoryview(f.read(length))
    if raw is None:
        raise ValueError(f"initializer {name} has no raw_data (typed data fields are not used by q4f16 exports)")
    return Tensor(name, dims, dtype, raw)


def read_initializers(path: str) -> Dict[str, Tensor]:
    """Every initializer of the model's graph, by name."""
    with open(path, "rb") as f:
        data = memoryview(f.read())
    graph = None
    for field, wt, v in _fields(data):
        if field == 7 and wt == 2:           # ModelProto.graph
            graph = v
    if graph is None:
        raise ValueError(f"{path}: no graph in the ONNX model")
    out: Dict[str, Tensor] = {}
    model_dir = os.path.dirname(os.path.abspath(path))
    for field, wt, v in _fields(graph):
        if field == 5 and wt == 2:           # GraphProto.initializer
            t = _tensor(v, model_dir)
            out[t.name] = t
    return out


# ---- extraction ---------------------------------------------------------------------

def _f16_to_f32(t: Tensor) -> np.ndarray:
    if t.data_type != FLOAT16:
        raise ValueError(f"Expected FLOAT16 tensor, got dataType={t.data_type} ({t.name})")
    return np.frombuffer(t.raw, dtype="<f2").astype(np.float32)


def extract_runtime(onnx_path: str, out_dir: str, layers: Optional[int] = None) -> dict:
    """Write the runtime directory for `onnx_path` into `out_dir`; returns the manifest.
    `layers` defaults to every layer the export holds."""
    inits = read_initializers(onnx_path)

    def need(name: str) -> Tensor:
        if name not in inits:
            raise KeyError(f"Missing initializer {name}")
        return inits[name]

    def write(rel: str, data) -> None:
        path = os.path.join(out_dir, rel)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "wb") as f:
            f.write(data)

    def entry(name: str, rel: str) -> dict:
        t = need(name)
        return {"name": name, "file": rel, "dims": [int(d) for d in t.dims], "dataType": t.data_type,
                "bytes": t.nbytes}

    def raw(name: str, rel: str) -> dict:
        write(rel, bytes(need(name).raw))
        return entry(name, rel)

    if layers is None:
        layers = 0
        while f"model.layers.{layers}.input_layernorm.weight" in inits:
            layers += 1
    embed = need("model.embed_tokens.weight")
    head_dim = int(need("model.layers.0.attn.q_norm.layernorm.weight").dims[0])
    q_out = int(need("model.layers.0.attn.q_proj.MatMul.weight_Q4").dims[0])
    k_out = int(need("model.layers.0.attn.k_proj.MatMul.weight_Q4").dims[0])
    manifest: dict = {
        "source": onnx_path,
        "dtype": "q4f16",
        "hiddenSize": int(embed.dims[1]),
        "intermediateSize": int(need("model.layers.0.mlp.gate_proj.MatMul.weight_Q4").dims[0]),
        "attentionHeads": q_out // head_dim,
        "kvHeads": k_out // head_dim,
        "headDim": head_dim,
        "layers": [],
        "shared": {},
        "finalNorm": None,
    }
    manifest["shared"]["embedTokens"] = raw("model.embed_tokens.weight", "shared/embed_tokens.f16")
    manifest["shared"]["cosCache"] = raw("cos_cache", "shared/cos_cache.f16")
    manifest["shared"]["sinCache"] = raw("sin_cache", "shared/sin_cache.f16")
    final = f"model.layers.{layers}.final_norm_layernorm.weight"
    manifest["finalNorm"] = raw(final, "shared/final_norm.f16")

    for layer in range(layers):
        d = f"layers/{layer}"
        le: dict = {"layer": layer, "norms": {}, "projections": {}}
        for key, suffix in NORMS:
            le["norms"][key] = raw(f"model.layers.{layer}.{suffix}", f"{d}/norm_{key}.f16")
        for key, suffix in PROJECTIONS:
            prefix = f"model.layers.{layer}.{suffix}"
            wname, sname = f"{prefix}.weight_Q4", f"{prefix}.weight_scales"
            w, s = need(wname), need(sname)
            wf, sf = f"{d}/{key}_weight_q4.bin", f"{d}/{key}_scales_f32.bin"
            write(wf, bytes(w.raw))
            scales = _f16_to_f32(s)
            write(sf, scales.tobytes())
            n, bpr, bpb = (int(x) for x in w.dims)
            le["projections"][key] = {
                "prefix": prefix,
                "weight": entry(wname, wf),
                "scales": {**entry(sname, sf), "sourceDataType": s.data_type, "dataType": "float32",
                           "bytes": scales.size * 4},
                "matmulNBits": {"outSize": n, "blocksPerRow": bpr, "bytesPerBlock": bpb, "blockSize": bpb * 2,
                                "inSize": bpr * bpb * 2},
            }
        manifest["layers"].append(le)

    os.makedirs(out_dir, exist_ok=True)
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        f.write(json.dumps(manifest, indent=2) + "\n")
    return manifest


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) < 2:
        print(__doc__.strip().splitlines()[-1].strip(), file=sys.stderr)
        return 2
    m = extract_runtime(argv[0], argv[1], int(argv[2]) if len(argv) > 2 else None)
    print(f"wrote {argv[1]}/manifest.json")
    print(f"layers={len(m['layers'])}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
