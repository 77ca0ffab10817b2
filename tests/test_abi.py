"""CPU tests of the C ABI boundary and the host-side API (no GPU needed)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from rustane_b200 import bridge as B
from rustane_b200.model import CONFIGS, ModelConfig

HEADER = Path(__file__).resolve().parents[1] / "include" / "cuda_bridge.h"


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(cb_\w+)\(", text, re.M)))


def test_header_declares_exported_list():
    assert header_functions() == sorted(B.EXPORTED)


def test_library_exports_every_declared_symbol(bridge_lib):
    for name in header_functions():
        assert hasattr(bridge_lib, name), name


def _header_arity():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(cb_\w+)\s*\(([^)]*)\)\s*;", text):
        params = [p for p in (x.strip() for x in m.group(2).split(",")) if p and p != "void"]
        out[m.group(1)] = len(params)
    return out


RUST_FFI = HEADER.parents[1] / "crates" / "cuda-bridge" / "src" / "lib.rs"


def test_python_and_rust_bindings_match_header_arity(bridge_lib):
    """The ctypes table (rustane_b200/bridge.py) and the extern block of the Rust
    cuda-bridge crate (crates/cuda-bridge/src/lib.rs) declare every entry point with
    the header's parameter count."""
    arity = _header_arity()
    assert sorted(arity) == header_functions()
    for name, n in arity.items():
        assert len(getattr(bridge_lib, name).argtypes) == n, name
    rust = RUST_FFI.read_text()
    block = rust[rust.index('unsafe extern "C" {'):]
    block = block[:block.index("\n    }\n")]
    bound = {m.group(1): len([p for p in m.group(2).split(",") if p.strip()])
             for m in re.finditer(r"pub fn (cb_\w+)\(([^)]*)\)", block)}
    assert bound == arity


def test_rust_crate_layout():
    """The crate that replaces crates/ane-bridge: a manifest with the workspace's
    package values, a build script that runs nvcc for sm_100a, and the library."""
    crate = RUST_FFI.parents[1]
    manifest = (crate / "Cargo.toml").read_text()
    assert 'name = "cuda-bridge"' in manifest and 'edition = "2024"' in manifest
    build = (crate / "build.rs").read_text()
    assert "arch=compute_100a,code=sm_100a" in build and "bridge.cu" in build
    assert "cargo:rustc-link-lib=dylib=cudabridge" in build


def test_version(bridge_lib):
    assert b"sm_100a" in bridge_lib.cb_version()


def test_device_count(bridge_lib):
    n = C.c_int32(-1)
    assert bridge_lib.cb_device_count(C.byref(n)) == B.CB_OK
    assert n.value >= 0


def _create(cfg_tuple, max_batch=1):
    lib = B.load_library()
    h = C.c_void_p()
    cfg = B.cb_model_config(*cfg_tuple)
    return lib.cb_create(C.byref(cfg), 0, max_batch, C.byref(h)), h


@pytest.mark.parametrize("bad", [
    (1536, 4096, 12, 12, 64, 512, 20, 8192),   # hd != 128
    (1500, 4096, 12, 12, 128, 512, 20, 8192),  # dim not a multiple of 256
    (1536, 4096, 12, 5, 128, 512, 20, 8192),   # heads % kv_heads
    (1536, 4096, 12, 12, 128, 500, 20, 8192),  # seq % 64
    (1536, 4096, 12, 12, 128, 512, 0, 8192),   # no layers
    (1536, 4000, 12, 12, 128, 512, 20, 8192),  # hidden % 64
])
def test_create_rejects_invalid_config(bridge_lib, bad):
    rc, h = _create(bad)
    assert rc == B.CB_ERR_INVALID_ARG
    assert not h.value
    assert bridge_lib.cb_create_error()


def test_create_rejects_bad_batch(bridge_lib):
    rc, _ = _create((256, 512, 2, 2, 128, 64, 1, 512), max_batch=0)
    assert rc == B.CB_ERR_INVALID_ARG


def test_create_without_gpu_fails_loudly(bridge_lib):
    n = C.c_int32()
    bridge_lib.cb_device_count(C.byref(n))
    if n.value > 0:
        pytest.skip("a GPU is present")
    rc, h = _create((256, 512, 2, 2, 128, 64, 1, 512))
    assert rc == B.CB_ERR_UNSUPPORTED
    assert b"no CUDA device" in bridge_lib.cb_create_error()


def test_null_context_calls_are_rejected(bridge_lib):
    assert bridge_lib.cb_destroy(None) == B.CB_OK
    assert bridge_lib.cb_init_weights(None, 0, 0, 0.02) == B.CB_ERR_INVALID_ARG
    assert bridge_lib.cb_forward_loss(None, None, None, 1, 0.0, None, None) == B.CB_ERR_INVALID_ARG
    assert bridge_lib.cb_gemm_f16(None, None, None, 128, 128, 64, 0, 0, None) == B.CB_ERR_INVALID_ARG
    assert bridge_lib.cb_last_error(None) == b"null context"


_NULL_OK = {"cb_destroy", "cb_tokens_close"}          # releasing nothing is fine
_STRINGS = {"cb_version", "cb_create_error", "cb_last_error"}


@pytest.mark.parametrize("name", sorted(B.EXPORTED))
def test_every_entry_point_rejects_null_arguments(bridge_lib, name):
    """Every call returns a status (never aborts, as the boundary promises): with null
    pointers and zero sizes each one answers CB_ERR_INVALID_ARG, without touching a
    device."""
    fn = getattr(bridge_lib, name)
    args = [0 if a in (C.c_int32, C.c_int64, C.c_uint32, C.c_uint64) else 0.0 if a is C.c_float else None
            for a in fn.argtypes]
    r = fn(*args)
    if name in _STRINGS:
        assert isinstance(r, bytes)
    elif name in _NULL_OK:
        assert r == B.CB_OK
    else:
        assert r == B.CB_ERR_INVALID_ARG, (name, r)


def test_python_api_raises_without_gpu(bridge_lib):
    n = C.c_int32()
    bridge_lib.cb_device_count(C.byref(n))
    if n.value > 0:
        pytest.skip("a GPU is present")
    from rustane_b200 import CompiledKernels, CudaBridgeError
    with pytest.raises(CudaBridgeError):
        CompiledKernels.compile_forward_only(ModelConfig.gpt_karpathy())


def test_param_counts_match_reference_presets():
    # model.rs doc comments: 600M ~579M, gpt_karpathy 48.8M incl. embedding
    assert abs(ModelConfig.target_600m().param_count() / 1e6 - 579) < 1
    assert CONFIGS["600m-A"] == ModelConfig.target_600m()


def test_flop_model_matches_the_per_forward_figures():
    """Algorithmic TFLOP per forward: 0.6088 for one 600m-A sequence of 512 tokens,
    2161 for the ~32B shape at 16 x 2048 tokens (2 x linear params + head + causal
    attention per token)."""
    cfg = CONFIGS["600m-A"]
    tflop_fwd = cfg.forward_flops_per_token() * 512 / 1e12
    assert abs(tflop_fwd - 0.6088) < 0.001
    c4 = CONFIGS["32B"]
    assert abs(c4.forward_flops_per_token() * 32768 / 1e12 - 2161.0) < 1.0


def test_bench_gemm_classes_exist_in_bridge():
    """bench.py's roofline sums these kernel classes; each must be a class the
    bridge reports (a rename must not silently drop a GEMM from the roofline)."""
    import importlib.util
    root = Path(__file__).resolve().parents[1]
    spec = importlib.util.spec_from_file_location("bench_mod", root / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    src = (root / "rustane_b200" / "csrc" / "bridge.cu").read_text()
    table = src[src.index("kclass_name"):src.index("kclass_name") + 800]
    for c in bench.GEMM_CLASSES:
        assert f'"{c}"' in table, c


def test_plain_c_client_compiles_links_and_runs(bridge_lib, tmp_path):
    """include/cuda_bridge.h is strict C99 (a Rust, cgo or C caller needs no C++), and a
    C program linked against the library gets status codes and messages back from the
    host-only calls (tests/c_abi_client.c)."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    root = HEADER.parents[1]
    lib_dir = root / "rustane_b200"
    exe = tmp_path / "c_abi_client"
    cc = subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                         f"-I{root / 'include'}", str(root / "tests" / "c_abi_client.c"),
                         f"-L{lib_dir}", "-lcudabridge", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "c client: ok" in run.stdout


def test_model_weights_touch_gives_a_new_generation():
    from rustane_b200 import ModelWeights
    w = ModelWeights.normal(CONFIGS["600m-A"], seed=1)
    g = w.generation
    w.touch()
    assert w.generation != g
