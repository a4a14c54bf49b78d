"""The C-ABI library loads without a GPU, exports every entry point include/*.h declares (and
the reference-named C++ entry points), and rejects bad arguments before touching CUDA."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

from nanochat_inferonly_lightning_b200 import _lib

HEADER = os.path.join(ROOT, "include", "nanochat_attn.h")
DROPIN = os.path.join(ROOT, "include", "nanochat_attn_dropin.hpp")


def declared_c_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"\b(nc_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def exported_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_loads():
    lib = _lib.load()
    assert lib.nc_status_string(0) == b"ok"


def test_every_declared_function_is_exported():
    names = declared_c_functions()
    assert len(names) >= 25
    syms = exported_symbols()
    missing = [n for n in names if n not in syms]
    assert not missing, missing
    # and the ctypes table covers exactly the header
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_dropin_cpp_symbols_exported():
    syms = exported_symbols()
    for name, mangled in _lib.DROPIN_SYMBOLS.items():
        assert mangled in syms, name
    # every function the drop-in header declares is one of them
    text = open(DROPIN).read()
    for fn in re.findall(r"^void (\w+)\(", text, flags=re.M):
        assert fn in _lib.DROPIN_SYMBOLS, fn


def test_dropin_mangling_matches_reference_declarations():
    """The mangled names are what src/model.h:14-16,26-27 declarations produce: compile a tiny
    translation unit with the reference's signatures and compare the symbols it references."""
    src = r'''
#include <cuda_runtime.h>
#include <cuda_bf16.h>
namespace nanochat {
void apply_rope(nv_bfloat16* x, int seq_len, int n_heads, int start_pos, cudaStream_t stream);
void apply_rope_rmsnorm(nv_bfloat16* x, int seq_len, int n_heads, int start_pos, cudaStream_t stream);
void init_rope_tables();
void flash_attention(nv_bfloat16* out, const nv_bfloat16* Q, const nv_bfloat16* K, const nv_bfloat16* V,
                     int seq_q, int kv_len, int heads, float scale, int kv_offset, cudaStream_t stream);
}
void use() {
  nanochat::apply_rope(0,0,0,0,0); nanochat::apply_rope_rmsnorm(0,0,0,0,0);
  nanochat::init_rope_tables(); nanochat::flash_attention(0,0,0,0,0,0,0,0.f,0,0);
}
'''
    import tempfile

    with tempfile.TemporaryDirectory() as d:
        cpp = os.path.join(d, "use.cpp")
        obj = os.path.join(d, "use.o")
        open(cpp, "w").write(src)
        subprocess.run(["g++", "-c", "-I/usr/local/cuda/include", cpp, "-o", obj], check=True)
        undef = subprocess.run(["nm", "-u", obj], capture_output=True, text=True).stdout
    wanted = {l.split()[-1] for l in undef.splitlines() if "nanochat" in l}
    assert wanted == set(_lib.DROPIN_SYMBOLS.values())


def test_argument_validation_without_gpu():
    lib = _lib.load()
    P = ctypes.c_void_p
    # negative sizes / bad head counts are rejected before any CUDA call
    assert lib.nc_flash_attention(P(256), P(256), P(256), P(256), -1, 4, 17, 0.1, 0, None) == 1
    assert lib.nc_flash_attention(P(256), P(256), P(256), P(256), 4, 4, 0, 0.1, 0, None) == 1
    assert lib.nc_flash_attention(P(256), P(256), P(256), P(256), 4, 4, 33, 0.1, 0, None) == 1
    # misaligned pointers
    assert lib.nc_flash_attention(P(258), P(256), P(256), P(256), 4, 4, 17, 0.1, 0, None) == 2
    assert lib.nc_apply_rope_rmsnorm(P(264), 4, 17, 0, None) == 2
    # positions beyond the RoPE table
    assert lib.nc_apply_rope_rmsnorm(P(256), 8, 17, 20480 - 4, None) == 5
    # zero-size calls are no-ops
    assert lib.nc_flash_attention(P(256), P(256), P(256), P(256), 0, 4, 17, 0.1, 0, None) == 0
    assert lib.nc_apply_rope(P(256), 0, 17, 0, None) == 0
    # decode: workspace required once there is more than one split
    assert lib.nc_decode_attention(P(256), P(256), None, None, P(256), P(256), P(256), 2, 17,
                                   0.1, 4096, 16, None, 0, None) == 4
    assert lib.nc_decode_attention(P(256), P(256), None, None, P(256), P(256), P(256), 2, 17,
                                   0.1, 4096, 24, None, 0, None) == 1  # split_len % 16
    # batched prefill: stride smaller than a sequence
    assert lib.nc_prefill_attention_batched(P(256), P(256), P(256), P(256), 100, 10, P(256), 2,
                                            4, 17, 0.1, None) == 1
    # KV cache creation with bad geometry
    h = ctypes.c_void_p()
    assert lib.nc_kv_cache_create(ctypes.byref(h), 0, 1, 16, 17) == 1
    assert lib.nc_kv_cache_create(ctypes.byref(h), 1, 1, 20481, 17) == 5
    for code in range(7):
        assert lib.nc_status_string(code) not in (b"", b"unknown status")


def test_gemm_argument_validation_without_gpu():
    """nc_gemm_skinny rejects bad sizes, flags, segments, alignment and aliasing before any
    CUDA call."""
    lib = _lib.load()
    P = ctypes.c_void_p
    F = ctypes.c_float

    def call(out=0x10000, x=0x20000, w=0x40000, res=None, M=8, N=2176, K=2176, flags=0,
             cap=0.0, seg=0, splits=0):
        return lib.nc_gemm_skinny(P(out), P(x), P(w), None if res is None else P(res), M, N,
                                  K, flags, F(cap), seg, splits, None)

    assert call(M=0) == 1 and call(M=65) == 1          # 1 <= M <= 64
    assert call(K=2180) == 1 and call(K=0) == 1         # K % 8 == 0, K >= 8
    assert call(N=0) == 1 and call(splits=-1) == 1
    assert call(flags=16) == 1                          # unknown flag
    assert call(flags=2) == 1                           # residual flag without a residual
    assert call(flags=8, cap=0.0) == 1                  # tanh cap needs cap > 0
    assert call(seg=1000) == 1                          # segment must divide N
    assert call(x=0x20008) == 2 and call(w=0x40004) == 2 and call(out=0x10001) == 2
    assert call(out=0x20000 + 64) == 1                  # out overlaps x
    assert call(res=0x10000 + 2, flags=2) == 1          # residual partly overlaps out


def test_step_ops_argument_validation_without_gpu():
    lib = _lib.load()
    P = ctypes.c_void_p
    assert lib.nc_embed_rmsnorm(P(256), P(256), P(256), 4, 2180, 100, None) == 1  # dim % 8
    assert lib.nc_embed_rmsnorm(P(256), P(256), P(256), 4, 16384, 100, None) == 1  # dim > 8192
    assert lib.nc_embed_rmsnorm(P(256), P(256), P(256), 4, 2176, 0, None) == 1    # vocab
    assert lib.nc_embed_rmsnorm(P(264), P(256), P(256), 4, 2176, 100, None) == 2  # alignment
    assert lib.nc_embed_rmsnorm(P(256), P(256), P(256), 0, 2176, 100, None) == 0  # empty
    assert lib.nc_argmax_rows(P(256), P(256), 4, 65530, None) == 1                 # cols % 8
    assert lib.nc_argmax_rows(P(256), P(264), 4, 65536, None) == 2
    assert lib.nc_argmax_rows(P(256), P(256), 0, 65536, None) == 0
    F = ctypes.c_float
    # sampling: top_k above 1024 with a filter, top_p <= 0, no draws or a negative temperature
    # are refused
    assert lib.nc_sample_rows(P(256), P(256), 4, 65536, F(1.0), 2000, F(0.9), P(256), None) == 1
    assert lib.nc_sample_rows(P(256), P(256), 4, 65536, F(1.0), 0, F(0.0), P(256), None) == 1
    # top-p over the whole row counts keys in 16 bits: vocab above 65536 is refused
    assert lib.nc_sample_rows(P(256), P(256), 4, 65544, F(1.0), 0, F(0.9), P(256), None) == 1
    assert lib.nc_sample_rows(P(256), P(256), 4, 65536, F(1.0), 50, F(0.9), None, None) == 1
    assert lib.nc_sample_rows(P(256), P(256), 4, 65536, F(-1.0), 50, F(0.9), P(256), None) == 1
