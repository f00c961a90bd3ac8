"""The drop-in boundary: libholo_cuda.so loads without a GPU and exports every
function declared in include/*.h, including every entry point of the
reference's include/cuda_ops.h; the two cuda_ops.h headers declare the same
types; the reference's own GPU host code links against the library.  CPU only
(no compute calls)."""
import ctypes
import os
import pathlib
import subprocess

import pytest

import holo_b200 as hb
from conftest import ROOT

DROPIN = ROOT / "oracle" / "_ref" / "libholo_ref_dropin.so"

# the 48 functions of the reference header include/cuda_ops.h (lines 18-133)
REFERENCE_ABI = """
cuda_init cuda_cleanup cuda_available cuda_print_info cuda_get_device_count cuda_get_free_memory
cuda_get_device_name cuda_malloc cuda_free cuda_memcpy_h2d cuda_memcpy_d2h cuda_memcpy_d2d
cuda_memcpy_d2d_async cuda_memcpy_d2h_async cuda_memset cuda_sync cuda_sync_copy cuda_vec_add
cuda_vec_mul cuda_vec_scale cuda_vec_dot cuda_matmul_f32 cuda_matmul_f16 cuda_matmul_q8_0
cuda_matmul_q4_0 cuda_matmul_q4_k cuda_matmul_q6_k cuda_batched_qkv_q8_0
cuda_batched_ffn_gate_up_q8_0 cuda_silu cuda_silu_mul cuda_gelu cuda_relu cuda_rms_norm
cuda_layer_norm cuda_softmax cuda_softmax_inplace cuda_attention_scores cuda_attention_apply
cuda_attention_single cuda_multi_head_attention cuda_rope_apply cuda_get_embedding_f32
cuda_get_embedding_f16 cuda_get_embedding_q8_0 cuda_get_embedding_q4_0 cuda_get_embedding_q6_k
cuda_argmax
""".split()


def exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(hb.LIB_PATH)], capture_output=True, text=True, check=True)
    return {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}


def test_library_loads_without_gpu(lib):
    assert lib is not None


def test_every_header_symbol_is_exported():
    names = hb.header_symbols()
    assert len(names) >= len(REFERENCE_ABI)
    missing = sorted(set(names) - exported())
    assert not missing, missing


def test_reference_abi_is_complete():
    declared = set(hb.header_symbols())
    assert len(REFERENCE_ABI) == 48
    assert set(REFERENCE_ABI) <= declared
    assert set(REFERENCE_ABI) <= exported()


def test_python_signatures_cover_headers():
    assert set(hb.header_symbols()) <= set(hb.SIGNATURES)


def test_kernels_are_built_for_sm100a_only():
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", str(hb.LIB_PATH)],
                         capture_output=True, text=True)
    archs = {w for w in out.stdout.split() if "sm_" in w}
    assert archs and all("sm_100a" in a for a in archs), archs


def test_reference_gpu_host_code_links_against_library():
    """The drop-in proof at link level: the reference's llm.c + llm_cuda.c,
    compiled as its CUDA build compiles them (HOLO_USE_CUDA) against this
    repository's include/cuda_ops.h, link against libholo_cuda.so in place of
    cuda_ops.cu with no undefined symbol (oracle/Makefile, target dropin).
    Every cuda_* function they call is a reference ABI function the library
    exports, and the linked library loads."""
    if not DROPIN.exists():
        pytest.skip("no drop-in build (the reference tree is absent)")
    out = subprocess.run(["nm", "-D", "--undefined-only", str(DROPIN)], capture_output=True, text=True, check=True)
    called = {line.split()[-1] for line in out.stdout.splitlines() if line.split()[-1].startswith("cuda_")}
    assert len(called) >= 20, called
    assert called <= set(REFERENCE_ABI), called - set(REFERENCE_ABI)
    assert called <= exported(), called - exported()
    ctypes.CDLL(str(DROPIN))


def reference_header():
    """include/cuda_ops.h of the reference tree that oracle/Makefile builds
    from: REF or HOLO_REFERENCE_DIR in the environment, else the checkout
    beside this repository (the Makefile's default)."""
    ref = os.environ.get("REF") or os.environ.get("HOLO_REFERENCE_DIR") or str(ROOT.parent / "reference")
    return pathlib.Path(ref) / "include" / "cuda_ops.h"


def compile_both(ours, tmp_path):
    """Compile one C file that includes the reference header and then ours:
    a prototype of ours that conflicts with the reference's is an error."""
    src = tmp_path / "both.c"
    src.write_text(f'#include "{reference_header()}"\n#undef HOLO_CUDA_OPS_H\n#include "{ours}"\n'
                   "int main(void) { return 0; }\n")
    return subprocess.run(["gcc", "-std=gnu11", "-Wall", "-Werror", "-c", str(src), "-o", str(tmp_path / "both.o")],
                          capture_output=True, text=True)


def test_header_prototypes_match_reference(tmp_path):
    """Type-level identity of the 48 declarations (names are checked above):
    the C compiler accepts the reference's and this build's header in one
    translation unit, and rejects a copy of ours with one parameter type
    changed."""
    if not reference_header().exists():
        pytest.skip("reference tree absent")
    ours = ROOT / "include" / "cuda_ops.h"
    p = compile_both(ours, tmp_path)
    assert p.returncode == 0, p.stderr
    bad = tmp_path / "cuda_ops_bad.h"
    text = ours.read_text()
    proto = "void cuda_matmul_q4_k(float *dst, const void *M, const float *v, int out_dim, int in_dim);"
    assert proto in text
    bad.write_text(text.replace(proto, proto.replace("int out_dim", "long out_dim")))
    p = compile_both(bad, tmp_path)
    assert p.returncode != 0 and "conflicting types" in p.stderr


@pytest.mark.parametrize("order", ["ours_first", "holo_first"])
def test_header_coexists_with_reference_holo_h(tmp_path, order):
    """A unit of the reference's app may include its holo.h (which declares
    HOLO_OK, HOLO_ERROR... as enumerators, include/holo.h:28-35) and this
    build's headers, in either order."""
    holo_h = reference_header().parent / "holo.h"
    if not holo_h.exists():
        pytest.skip("reference tree absent")
    ours = [f'#include "{ROOT / "include" / "cuda_ops.h"}"', f'#include "{ROOT / "include" / "holo_b200.h"}"']
    lines = ours + [f'#include "{holo_h}"'] if order == "ours_first" else [f'#include "{holo_h}"'] + ours
    src = tmp_path / "both.c"
    src.write_text("\n".join(lines) + "\nint main(void) { return HOLO_OK + HOLO_STATUS_OK; }\n")
    p = subprocess.run(["gcc", "-std=gnu11", "-Wall", "-Werror", "-c", str(src), "-o", str(tmp_path / "both.o")],
                       capture_output=True, text=True)
    assert p.returncode == 0, p.stderr
