"""Weight file format (preprocess_layer_fixed_gpu.py:245-282, binary_loader.hpp:59-193) and
the C ABI's symbol table.  No GPU needed."""
import os
import re

import numpy as np
import pytest

from conftest import ROOT, golden


def test_save_load_roundtrip(weights_mod, tmp_path):
    g = golden("bm_256x64.npz")
    bw = weights_mod.bucketize_fp16_packed(g["W"].view(np.float16))
    p = str(tmp_path / "layer0_q_proj_bucketmul_fp16")
    weights_mod.save_bucketmul_binary(bw, p)
    meta = open(p + "_meta.txt").read()
    assert "buckets_shape: 1 1024 16" in meta and "stats_shape: 1 1024 4" in meta
    assert "probes_shape: 1 64" in meta and "in_dim: 64" in meta and "out_dim: 256" in meta
    back = weights_mod.load_bucketmul_binary(p)
    np.testing.assert_array_equal(back.buckets, bw.buckets)
    np.testing.assert_array_equal(back.stats, bw.stats)
    np.testing.assert_array_equal(back.probes, bw.probes)
    assert (back.in_dim, back.out_dim, back.bsize) == (64, 256, 16)


@pytest.mark.parametrize("case", ["bm_256x64.npz", "bm_128x512.npz", "bm_48x96_ties.npz", "bm_16x4096.npz"])
def test_dense_unpack_restatement_on_reference_buckets(weights_mod, case):
    """The dense matrix behind the dense tensor-core path: unpacking the reference's own bucket
    layout (fixtures made by preprocess_layer_fixed_gpu.py) puts every packed word back at
    (16*c + slot, i), i.e. W with its row's slot in the low 4 mantissa bits."""
    g = golden(case)
    dense = weights_mod.dense_from_buckets(g["buckets"])
    assert dense.shape == g["W"].shape
    np.testing.assert_array_equal(dense, weights_mod.dense_packed(g["W"].view(np.float16)))


def test_truncated_file_is_rejected(weights_mod, tmp_path):
    g = golden("bm_256x64.npz")
    bw = weights_mod.bucketize_fp16_packed(g["W"].view(np.float16))
    p = str(tmp_path / "w")
    weights_mod.save_bucketmul_binary(bw, p)
    with open(p + "_stats.bin", "r+b") as f:
        f.truncate(100)
    with pytest.raises(weights_mod.WeightFormatError, match="File size mismatch"):
        weights_mod.load_bucketmul_binary(p)


def test_missing_files_and_dims(weights_mod, tmp_path):
    with pytest.raises(weights_mod.WeightFormatError, match="Cannot open metadata"):
        weights_mod.load_bucketmul_binary(str(tmp_path / "nope"))
    p = str(tmp_path / "bad")
    with open(p + "_meta.txt", "w") as f:
        f.write("# no dims\nbsize: 16\n")
    with pytest.raises(weights_mod.WeightFormatError, match="missing dimensions"):
        weights_mod.load_bucketmul_binary(p)


def test_npy_fp16_roundtrip(weights_mod, tmp_path):
    a = (np.arange(4096) * 0.001).astype(np.float16)
    p = str(tmp_path / "layer0_input_layernorm.npy")
    weights_mod.save_npy_fp16(p, a)
    np.testing.assert_array_equal(weights_mod.load_npy_fp16(p), a.view(np.uint16))


def _declared_symbols():
    syms = []
    for name in os.listdir(os.path.join(ROOT, "include")):
        if name.endswith(".h"):
            text = open(os.path.join(ROOT, "include", name)).read()
            syms += re.findall(r"^\s*(?:const\s+char\s*\*|int|void)\s+(iam_\w+)\s*\(", text, re.M)
    return sorted(set(syms))


def test_library_exports_every_declared_symbol(iam):
    """libiamb200.so loads without a GPU and exports every entry point include/*.h declares."""
    lib = iam.load_library()
    declared = _declared_symbols()
    assert declared, "no declarations found"
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    bound = set(iam.exported_symbols())
    assert bound <= set(declared) | {"iam_version", "iam_last_error"}, sorted(bound - set(declared))
    assert lib.iam_version().startswith(b"iam-b200")


def test_python_binding_covers_header(iam):
    assert set(_declared_symbols()) <= set(iam.exported_symbols()) | {"iam_model_forward_tokens"}


def test_cpp_shim_compiles(tmp_path):
    """include/iam_b200.hpp (the reference's class names over the C ABI) compiles as C++17."""
    import shutil
    import subprocess
    cuda_inc = "/usr/local/cuda/include"
    cxx = shutil.which("g++")
    if not cxx or not os.path.isdir(cuda_inc):
        pytest.skip("no host C++ compiler or CUDA headers")
    src = tmp_path / "shim.cpp"
    src.write_text('#include "iam_b200.hpp"\n'
                   'int main() {\n'
                   '  iam_model_config c = iam_shim::MistralModel::mistral7b(32000, 4096);\n'
                   '  return c.dim == 4096 ? 0 : 1;\n'
                   '}\n')
    r = subprocess.run([cxx, "-std=c++17", "-fsyntax-only", "-Wall", "-I", os.path.join(ROOT, "include"),
                        "-I", cuda_inc, str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
