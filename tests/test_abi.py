"""CPU-only checks of the C ABI and of the host-side logic (no GPU calls)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import oracle as O
from esolearn_b200 import _native as N
from esolearn_b200 import llama as LL

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_symbols():
    src = open(os.path.join(ROOT, "include", "sb_api.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sb_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = N.lib()
    syms = _header_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, f"declared in sb_api.h but not exported: {missing}"


def test_bindings_cover_the_header():
    assert sorted(N.SIGNATURES) == _header_symbols()


def test_abi_version_and_error_channel():
    lib = N.lib()
    assert lib.sb_abi_version() == 1
    # A call rejected on its arguments sets the error message without a GPU.
    rc = lib.sb_qweight_create(0, 0, 0, C.byref(C.c_void_p()))
    assert rc == 6
    assert "bad argument" in N.last_error()
    with pytest.raises(N.SbError):
        N.check(rc)


def test_config_struct_layout_matches_header(tmp_path):
    # Compile the header with the system C compiler and compare the layout of
    # sb_llama_config with the ctypes mirror field by field.
    fields = [f for f, _ in N.LlamaConfigC._fields_]
    prog = ['#include <stdio.h>', '#include <stddef.h>', '#include "sb_api.h"', 'int main(void) {',
            'printf("%zu\\n", sizeof(sb_llama_config));']
    prog += [f'printf("%zu\\n", offsetof(sb_llama_config, {f}));' for f in fields]
    prog += ['return 0; }']
    src = tmp_path / "layout.c"
    src.write_text("\n".join(prog))
    exe = tmp_path / "layout"
    import subprocess
    subprocess.run(["/usr/bin/gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert vals[0] == C.sizeof(N.LlamaConfigC)
    for f, off in zip(fields, vals[1:]):
        assert getattr(N.LlamaConfigC, f).offset == off, f


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_host_quantizer_bit_exact_vs_oracle(seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(10007) * 0.02).astype(np.float32)
    w[::97] = 0.0
    q, s = LL.quantize_symmetric(w)
    qo, so = O.quantize_symmetric(w)
    assert s == so and np.array_equal(q.ravel(), qo)


def test_host_quantizer_reference_tests():
    # quantize.rs:67-83
    q, s = LL.quantize_symmetric(np.zeros(10, np.float32))
    assert (q == 0).all() and s == 0.0
    q, _ = LL.quantize_symmetric(np.array([1000.0, -1000.0, 0.0], np.float32))
    assert q.tolist() == [127, -127, 0]


def test_sampler_rng_matches_oracle_rng():
    a, b = LL.Rng(123), O.Rng(123)
    for _ in range(50):
        assert a.f64() == b.f64()


@pytest.mark.parametrize("cfg", [
    LL.SamplingConfig(0.5, 5, 1.0, 4), LL.SamplingConfig(1.0, 0, 0.9, 4), LL.SamplingConfig(2.0, 10, 0.5, 4),
    LL.SamplingConfig(0.0, 0, 1.0, 4)])
def test_sample_token_matches_oracle(cfg):
    # generate.rs:92-165 restated twice (host package vs oracle) on the same draws.
    rng = np.random.default_rng(9)
    for t in range(20):
        logits = rng.standard_normal(300).astype(np.float32)
        ra, rb = LL.Rng(t), O.Rng(t)
        assert LL.sample_token(logits, cfg, ra) == O.sample_token(logits, cfg.temperature, cfg.top_k, cfg.top_p, rb)


def test_argmax_last_tie_rule():
    assert LL.argmax_last(np.array([1.0, 3.0, 3.0, 2.0], np.float32)) == 2
