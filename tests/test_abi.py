"""C-ABI checks that need no GPU: the library loads, exports every entry point
that include/kg_abi.h declares, and its host-side functions agree with the
oracle bit for bit (weights init, packed sizes)."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(kg_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    syms = declared_symbols()
    for must in ("kg_ctx_create", "kg_forward_token", "kg_forward_batch", "kg_tq_encode", "kg_kv_codes"):
        assert must in syms


def test_library_exports_every_declared_symbol(kg):
    lib = ctypes.CDLL(kg.LIBPATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_config_micro_defaults(kg):
    c = kg.micro_config()
    assert (c.vocab_size, c.block_size, c.n_embd, c.n_head, c.head_dim, c.n_kv_head,
            c.mlp_hidden, c.n_layer, c.bos_token) == (27, 16, 16, 4, 4, 4, 64, 1, 26)
    assert c.temperature == 0.5 and abs(c.sparse_threshold - 0.8) < 1e-7
    assert c.tq_seed == 42 and c.spkv_window == 128


@pytest.mark.parametrize("shape", [dict(), dict(n_layer=4), dict(n_layer=2, n_embd=32, n_head=4, head_dim=8,
                                                                   mlp_hidden=128, vocab_size=50)])
def test_reference_weights_match_oracle(kg, orc, shape):
    c = kg.micro_config(**shape)
    w = kg.reference_weights(c, seed=42)
    o = orc.weights(orc.from_kg(c), 42)
    assert w.shape == o.shape and np.array_equal(w, o)
    w2 = kg.reference_weights(c, seed=7, scale_mode=1, std=0.02)
    o2 = orc.weights(orc.from_kg(c), 7, 1, 0.02)
    assert np.array_equal(w2, o2)


def test_packed_len_matches_oracle(kg, orc):
    for dim in (1, 15, 16, 17, 768, 4096):
        for bits in (2, 3, 4, 5, 8):
            assert kg.lib().kg_tq_packed_len(dim, bits) == orc.packed_len(dim, bits)


def test_status_strings(kg):
    for s in range(-7, 1):
        assert kg.lib().kg_status_string(s)


def test_invalid_config_rejected_without_device(kg):
    c = kg.micro_config(n_head=3)  # n_head * head_dim != n_embd
    h = ctypes.c_void_p()
    rc = kg.lib().kg_ctx_create(ctypes.byref(c), 0, ctypes.byref(h))
    assert rc == -1 and not h


def test_cpp_trait_mirror_compiles(tmp_path):
    """include/kg_backend.hpp (the C++ InferenceBackend mirror) compiles against kg_abi.h."""
    import subprocess
    src = tmp_path / "t.cpp"
    src.write_text('#include "kg_backend.hpp"\n'
                   'int main() { kg_config c; kg_config_micro(&c); katgpt::CudaBackend b(c); '
                   'b.reset(); return b.is_compiled() ? 0 : 1; }\n')
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", os.path.join(ROOT, "include"), str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def _header_prototypes():
    src = open(os.path.join(ROOT, "include", "kg_abi.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    protos = {}
    for m in re.finditer(r"\b(kg_\w+)\s*\(([^;{]*?)\)\s*;", src, re.S):
        args = [a for a in " ".join(m.group(2).split()).split(",") if a.strip()]
        protos[m.group(1)] = len(args)
    return protos


def _header_struct_fields(name):
    src = open(os.path.join(ROOT, "include", "kg_abi.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    body = re.search(r"typedef struct \{([^}]*)\}\s*" + name + ";", src).group(1)
    return re.findall(r"\b(\w+)\s*;", body)


def test_rust_binding_matches_header():
    # the Rust -sys block a maintainer would add binds every entry point with
    # the header's parameter count, and its structs carry the header's fields in order
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    rust = doc[doc.index("```rust"):]
    rust = rust[:rust.index("```", 7)]
    bound = {m.group(1): len([a for a in " ".join(m.group(2).split()).split(",") if a.strip()])
             for m in re.finditer(r"pub fn (kg_\w+)\(([^)]*)\)", rust, re.S)}
    assert bound == _header_prototypes()
    for c, r in (("kg_config", "KgConfig"), ("kg_sq_params", "KgSqParams")):
        body = re.search(r"pub struct " + r + r" \{([^}]*)\}", rust).group(1)
        assert re.findall(r"pub (\w+):", body) == _header_struct_fields(c), c


def test_python_mirror_signatures_match_header(kg):
    # every entry point is bound in kgcuda with the header's parameters: same
    # count, pointers as pointers, scalars of the same width and kind (an
    # int32 bound where the C side reads int64 would pass garbage high bits)
    src = open(os.path.join(ROOT, "include", "kg_abi.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    scalar = {"int32_t": ctypes.c_int32, "int": ctypes.c_int, "int64_t": ctypes.c_int64,
              "uint64_t": ctypes.c_uint64, "float": ctypes.c_float}

    def same(c_type, t):
        if "*" in c_type:
            return t in (ctypes.c_void_p, ctypes.c_char_p) or issubclass(t, ctypes._Pointer)
        if c_type == "void":
            return t is None
        want = scalar[c_type.replace("const ", "").strip()]
        return ctypes.sizeof(t) == ctypes.sizeof(want) and (t is ctypes.c_float) == (want is ctypes.c_float)

    L = kg.lib()
    protos = list(re.finditer(r"([\w \*]+?)\b(kg_\w+)\s*\(([^;{]*?)\)\s*;", src, re.S))
    assert len(protos) == len(_header_prototypes())
    for m in protos:
        name = m.group(2)
        args = [a.strip() for a in " ".join(m.group(3).split()).split(",") if a.strip()]
        fn = getattr(L, name)
        assert fn.argtypes is not None and len(fn.argtypes) == len(args), name
        for a, t in zip(args, fn.argtypes):
            c_type = a if "*" in a else a.rsplit(" ", 1)[0]
            assert same(c_type, t), (name, a, t)
        ret = " ".join(m.group(1).split())
        if "*" not in ret and ret != "void":
            assert same(ret, fn.restype), (name, ret, fn.restype)
