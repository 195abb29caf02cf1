"""Real-weight ingest (onnx_ingest, restating scripts/extract-qwen-runtime-assets.mjs):
a q4f16 ONNX model written here from seeded synthetic weights must extract to the same
runtime files, byte for byte, that the synthetic generator writes, and the oracle
must decode identically from both directories. No GPU needed."""
import json
import os

import numpy as np
import pytest

from kernel_optimization_webgpu_b200 import onnx_ingest, synth
from oracle import oracle as O


# ---- a minimal protobuf writer for the test model -----------------------------------

def _varint(n: int) -> bytes:
    out = bytearray()
    while True:
        b = n & 0x7F
        n >>= 7
        out.append(b | (0x80 if n else 0))
        if not n:
            return bytes(out)


def _field(num: int, wt: int, payload) -> bytes:
    key = _varint((num << 3) | wt)
    if wt == 0:
        return key + _varint(payload)
    return key + _varint(len(payload)) + payload


def _tensor(name, dims, dtype, raw=None, external=None) -> bytes:
    msg = _field(1, 2, b"".join(_varint(d) for d in dims)) + _field(2, 0, dtype) + _field(8, 2, name.encode())
    if external is None:
        msg += _field(9, 2, raw)
    else:
        for k, v in external.items():
            msg += _field(13, 2, _field(1, 2, k.encode()) + _field(2, 2, str(v).encode()))
        msg += _field(14, 0, 1)
    return msg


def write_onnx(runtime_dir: str, path: str, external_name: str = None) -> None:
    """An ONNX model whose initializers hold the runtime directory's tensors under the
    export's names (f16 scales, q4 weights [N][K/32][16]); `external_name` is stored
    as external data in a side file."""
    m = json.load(open(os.path.join(runtime_dir, "manifest.json")))
    rd = lambda e: open(os.path.join(runtime_dir, e["file"]), "rb").read()  # noqa: E731
    inits = []
    side = bytearray()

    def add(name, dims, dtype, raw):
        if name == external_name:
            inits.append(_tensor(name, dims, dtype, external={"location": "weights.bin", "offset": len(side),
                                                             "length": len(raw)}))
            side.extend(raw)
        else:
            inits.append(_tensor(name, dims, dtype, raw))

    sh = m["shared"]
    add("model.embed_tokens.weight", sh["embedTokens"]["dims"], 10, rd(sh["embedTokens"]))
    add("cos_cache", sh["cosCache"]["dims"], 10, rd(sh["cosCache"]))
    add("sin_cache", sh["sinCache"]["dims"], 10, rd(sh["sinCache"]))
    L = len(m["layers"])
    add(f"model.layers.{L}.final_norm_layernorm.weight", m["finalNorm"]["dims"], 10, rd(m["finalNorm"]))
    names = dict(onnx_ingest.NORMS)
    for le in m["layers"]:
        i = le["layer"]
        for key, e in le["norms"].items():
            add(f"model.layers.{i}.{names[key]}", e["dims"], 10, rd(e))
        for key, suffix in onnx_ingest.PROJECTIONS:
            p = le["projections"][key]
            nb = p["matmulNBits"]
            add(f"model.layers.{i}.{suffix}.weight_Q4", [nb["outSize"], nb["blocksPerRow"], 16], 2, rd(p["weight"]))
            scales = np.frombuffer(rd(p["scales"]), np.float32).astype(np.float16)
            add(f"model.layers.{i}.{suffix}.weight_scales", [scales.size], 10, scales.tobytes())
    graph = b"".join(_field(5, 2, t) for t in inits)
    with open(path, "wb") as f:
        f.write(_field(1, 0, 8) + _field(7, 2, graph))
    if side:
        with open(os.path.join(os.path.dirname(path), "weights.bin"), "wb") as f:
            f.write(bytes(side))


@pytest.fixture(scope="module")
def tiny_onnx(tmp_path_factory, tiny_runtime):
    d = tmp_path_factory.mktemp("onnx")
    path = str(d / "model_q4f16.onnx")
    write_onnx(tiny_runtime, path, external_name="model.layers.1.mlp.down_proj.MatMul.weight_Q4")
    return path


def test_extracts_the_same_runtime_files(tiny_runtime, tiny_onnx, tmp_path):
    out = str(tmp_path / "runtime")
    m = onnx_ingest.extract_runtime(tiny_onnx, out)
    want = json.load(open(os.path.join(tiny_runtime, "manifest.json")))
    s = synth.TINY
    assert (m["hiddenSize"], m["intermediateSize"], m["attentionHeads"], m["kvHeads"], m["headDim"]) == \
        (s.hidden, s.intermediate, s.heads, s.kv_heads, s.head_dim)
    assert len(m["layers"]) == s.layers == len(want["layers"])
    files = [want["shared"][k]["file"] for k in ("embedTokens", "cosCache", "sinCache")] + [want["finalNorm"]["file"]]
    for le in want["layers"]:
        files += [e["file"] for e in le["norms"].values()]
        for p in le["projections"].values():
            files += [p["weight"]["file"], p["scales"]["file"]]
    for rel in files:
        a = open(os.path.join(tiny_runtime, rel), "rb").read()
        b = open(os.path.join(out, rel), "rb").read()
        assert a == b, rel
    for le_got, le_want in zip(m["layers"], want["layers"]):
        for key in le_want["projections"]:
            assert le_got["projections"][key]["matmulNBits"] == le_want["projections"][key]["matmulNBits"]
            assert le_got["projections"][key]["scales"]["dataType"] == "float32"


def test_oracle_decodes_the_same_from_the_extracted_runtime(tiny_runtime, tiny_onnx, tmp_path):
    out = str(tmp_path / "runtime")
    onnx_ingest.extract_runtime(tiny_onnx, out)
    prompt = [5, 77, 1000, 3]
    a = O.Model(tiny_runtime).session(max_seq=32).greedy(prompt, 6)
    b = O.Model(out).session(max_seq=32).greedy(prompt, 6)
    assert a[0] == b[0] and np.array_equal(a[1], b[1])


def test_rejects_a_model_without_the_expected_initializers(tmp_path):
    path = str(tmp_path / "empty.onnx")
    with open(path, "wb") as f:
        f.write(_field(1, 0, 8) + _field(7, 2, _field(5, 2, _tensor("x", [1], 10, b"\0\0"))))
    with pytest.raises(KeyError, match="model.embed_tokens.weight"):
        onnx_ingest.extract_runtime(path, str(tmp_path / "out"), layers=1)
    with open(path, "wb") as f:
        f.write(_field(1, 0, 8))
    with pytest.raises(ValueError, match="no graph"):
        onnx_ingest.read_initializers(path)


@pytest.mark.gpu
def test_engine_decodes_the_extracted_runtime(tiny_runtime, tiny_onnx, tmp_path):
    """The CUDA engine loads the extracted directory and emits the oracle's greedy ids."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernel_optimization_webgpu_b200 import runtime as R
    out = str(tmp_path / "runtime")
    onnx_ingest.extract_runtime(tiny_onnx, out)
    prompt = [5, 77, 1000, 3]
    want, _ = O.Model(tiny_runtime).session(max_seq=32).greedy(prompt, 6)
    with R.Engine(out, max_seq=32) as eng:
        ids, _ = eng.generate_greedy(prompt, 6)
    assert ids == want
