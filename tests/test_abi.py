"""The C-ABI library: builds, loads, exports what include/qdecode.h declares, and
rejects bad input on the host (no GPU needed for any of these)."""
import ctypes as C
import json
import os
import re

import pytest

from kernel_optimization_webgpu_b200 import _lib, runtime, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "qdecode.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qd_[a-z0-9_]+)\s*\(", text)) - {"qd_token_cb"})


def test_library_exports_every_declared_function():
    L = _lib.load()
    declared = header_functions()
    assert declared, "no declarations parsed"
    missing = [f for f in declared if not hasattr(L, f)]
    assert not missing, missing
    assert sorted(_lib.EXPORTS) == declared


def test_library_loads_without_torch():
    """Loading libqdecode.so alone (a fresh interpreter that never imports torch)
    maps no libtorch / libc10: the library is plain C ABI over the CUDA runtime."""
    import subprocess
    import sys
    code = ("import ctypes, sys; ctypes.CDLL(sys.argv[1]); "
            "maps = open('/proc/self/maps').read(); "
            "bad = [n for n in ('libtorch', 'libc10') if n in maps]; "
            "print('loaded'); sys.exit(1 if bad else 0)")
    _lib.load()  # builds the library when its sources are newer
    res = subprocess.run([sys.executable, "-c", code, _lib.lib_path()], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0 and "loaded" in res.stdout, res.stdout + res.stderr


def test_build_recipe_targets_sm100a_only():
    from kernel_optimization_webgpu_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_options_default():
    opt = _lib.QdOptions()
    _lib.load().qd_options_default(C.byref(opt))
    assert opt.max_seq == 256 and opt.kv_dtype == _lib.QD_KV_F16 and opt.use_graph == 1
    assert opt.rope_row_stride == 0 and opt.variant == b"optimized"
    assert opt.persistent == 1 and opt.timeline == 0 and opt.prompt_pass == 1


def _create(runtime_dir, **kw):
    return runtime.Engine(runtime_dir, **kw)


def test_create_rejects_missing_runtime(tmp_path):
    with pytest.raises(_lib.QdError) as ex:
        _create(str(tmp_path / "nope"))
    assert ex.value.code == _lib.QD_E_IO
    assert "manifest.json" in str(ex.value)


def test_create_rejects_malformed_manifest(tmp_path):
    (tmp_path / "manifest.json").write_text("{\"hiddenSize\": 1024, ")
    with pytest.raises(_lib.QdError) as ex:
        _create(str(tmp_path))
    assert ex.value.code == _lib.QD_E_IO


def _manifest_copy(src_dir, dst_dir, edit):
    m = json.load(open(os.path.join(src_dir, "manifest.json")))
    edit(m)
    os.makedirs(dst_dir, exist_ok=True)
    json.dump(m, open(os.path.join(dst_dir, "manifest.json"), "w"))


def test_create_rejects_unsupported_head_dim(tiny_runtime, tmp_path):
    _manifest_copy(tiny_runtime, str(tmp_path), lambda m: m.update(headDim=64))
    with pytest.raises(_lib.QdError) as ex:
        _create(str(tmp_path))
    assert ex.value.code in (_lib.QD_E_INVALID, _lib.QD_E_IO)


def test_create_rejects_projection_shape_mismatch(tiny_runtime, tmp_path):
    def edit(m):
        m["layers"][1]["projections"]["down"]["matmulNBits"]["outSize"] = 7
    _manifest_copy(tiny_runtime, str(tmp_path), edit)
    with pytest.raises(_lib.QdError) as ex:
        _create(str(tmp_path))
    assert ex.value.code == _lib.QD_E_IO and "down" in str(ex.value)


def test_create_rejects_block_size_other_than_32(tiny_runtime, tmp_path):
    def edit(m):
        d = m["layers"][0]["projections"]["q"]["matmulNBits"]
        d["blockSize"], d["blocksPerRow"] = 64, d["blocksPerRow"] // 2
    _manifest_copy(tiny_runtime, str(tmp_path), edit)
    with pytest.raises(_lib.QdError):
        _create(str(tmp_path))


def test_create_rejects_max_seq_beyond_rope_table(tiny_runtime):
    # TINY has 4096 table rows; position p reads row 2p, so 2049 positions do not fit.
    with pytest.raises(_lib.QdError) as ex:
        _create(tiny_runtime, max_seq=2049)
    assert ex.value.code == _lib.QD_E_RANGE


def test_kernel_entry_points_validate_before_touching_the_device():
    L = _lib.load()
    p = C.c_void_p(16)
    assert L.qd_q4_matvec(p, p, p, p, 1024, 8, 32, 16, None) == _lib.QD_E_INVALID   # block 16
    assert L.qd_q4_matvec(p, p, p, p, 2048, 8, 32, 32, None) == _lib.QD_E_INVALID   # in_size > 32*32
    assert L.qd_q4_matvec(None, p, p, p, 1024, 8, 32, 32, None) == _lib.QD_E_INVALID
    assert b"block_size" in L.qd_last_error(None) or L.qd_last_error(None)
    assert L.qd_lm_head_argmax(p, None, 1e-6, p, None, p, 1000, 10, p, None) == _lib.QD_E_INVALID
    assert L.qd_gqa_decode(p, p, p, 0, p, 10, 16, 8, 64, p, None) == _lib.QD_E_INVALID
    assert L.qd_gqa_decode(p, p, p, 0, p, 10, 15, 8, 128, p, None) == _lib.QD_E_INVALID
    assert L.qd_lm_head_argmax_workspace_bytes(151936) >= 256 + 8 * 148
    assert L.qd_gqa_decode_workspace_bytes(2048, 16) >= 8 * 16 * (128 * 4 + 8)


def test_greedy_api_rejects_over_long_requests_like_the_reference():
    dev = runtime.CudaDevice("/nonexistent")
    with pytest.raises(ValueError, match="up to 256 tokens"):
        runtime.runCustomQwenGreedyPrompt(device=dev, profile=runtime.qwenProfile,
                                          inputIds=list(range(200)), maxNewTokens=57)


def test_qwen_profile_mirrors_the_reference_profile():
    p = runtime.qwenProfile
    s = synth.QWEN3_0_6B
    assert (p["layers"], p["hiddenSize"], p["intermediateSize"], p["attentionHeads"], p["kvHeads"],
            p["headDim"], p["vocabSize"], p["normEpsilon"]) == (s.layers, s.hidden, s.intermediate, s.heads,
                                                               s.kv_heads, s.head_dim, s.vocab, s.eps)


def test_bindings_match_the_declared_arity():
    """Every ctypes binding passes exactly as many arguments as its C declaration
    takes (a mismatch would pass garbage through the ABI without any error)."""
    text = open(os.path.join(ROOT, "include", "qdecode.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = dict(re.findall(r"\b(qd_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S))
    decls.pop("qd_token_cb", None)
    assert set(decls) == set(header_functions())
    L = _lib.load()
    for name, params in decls.items():
        p = params.strip()
        n = 0 if p in ("", "void") else len(p.split(","))
        argtypes = getattr(L, name).argtypes
        assert argtypes is not None, name
        assert len(argtypes) == n, (name, n, len(argtypes))


def test_bindings_match_the_declared_return_types():
    """size_t results come back as 64-bit values, strings as char pointers, void as None."""
    text = open(os.path.join(ROOT, "include", "qdecode.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    want = {"int": C.c_int, "size_t": C.c_size_t, "const char*": C.c_char_p, "void": None}
    L = _lib.load()
    seen = 0
    for ret, name in re.findall(r"(int|size_t|const char\s*\*|void)\s+(qd_[a-z0-9_]+)\s*\(", text):
        ret = re.sub(r"\s+", "", ret).replace("constchar*", "const char*")
        assert getattr(L, name).restype is want[ret], (name, ret)
        seen += 1
    assert seen == len(header_functions())


def test_js_shim_exports_the_reference_functions():
    """The JS shim exports the four functions of src/bench/webgpu-runtime.js that callers
    import (createWebGpuContext, runKernelBenchmarks, runFullDecoderStackBenchmark,
    runCustomQwenGreedyPrompt), and the addon registers every native call the shim uses."""
    js = open(os.path.join(ROOT, "kernel_optimization_webgpu_b200", "js", "cuda-runtime.js")).read()
    exported = set(re.findall(r"export async function (\w+)", js))
    assert exported == {"createWebGpuContext", "runKernelBenchmarks", "runFullDecoderStackBenchmark",
                        "runCustomQwenGreedyPrompt"}
    used = set(re.findall(r"native\.(\w+)\(", js))
    addon = open(os.path.join(ROOT, "kernel_optimization_webgpu_b200", "js", "addon.cc")).read()
    registered = set(re.findall(r'\{"(\w+)", nullptr,', addon))
    assert used and used <= registered, used - registered
