"""The exact micro forward kernel's own source (katgpt-rs_b200/csrc/
kg_micro_kernel.cuh) run on host threads, one per CUDA thread of a block with
a barrier for __syncthreads (tests/host/micro_forward_host.cpp), against the
oracle on the CPU: forward_base teacher-forced over 16 positions, with and
without a writer LoRA adapter; forward_prefill followed by single-token
decode steps at 1 and 8 layers, with the LoraPair's reader and writer;
forward_quantized over 3- and 4-bit TurboQuant codes; forward_paged with pages
out of order in the pool (the pool's K/V rows compared too); and
forward_quantized over the SpectralQuant codec, uniform and water-filled
widths; and forward_sp_kv_quant with and without the writer adapter. Bar:
bit-identical logits (forward_sp_kv_quant: layer-0 codes and norms
bit-identical, logits within 1e-5 relative, as its GPU tests). The GPU tests run the same source compiled
for sm_100a."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CASES = 15


def test_micro_kernel_source_matches_oracle_on_host(orc, tmp_path):
    lib = orc.lib()
    libdir = os.path.dirname(lib._name)
    exe = tmp_path / "micro_forward_host"
    cmd = ["g++", "-O2", "-std=c++20", "-ffp-contract=off", "-fno-fast-math", "-pthread", "-Wno-unknown-pragmas",
           "-I", os.path.join(ROOT, "katgpt-rs_b200", "csrc"), "-I", os.path.join(ROOT, "oracle"),
           os.path.join(ROOT, "tests", "host", "micro_forward_host.cpp"), "-L", libdir, "-lkgoracle",
           "-Wl,-rpath," + libdir, "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        pytest.fail(r.stderr[-3000:])
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True, timeout=300).stdout.split("\n")
    rows = [tuple(map(int, ln.split())) for ln in out if ln.strip()]
    assert len(rows) == CASES
    for case, (bad, total) in enumerate(rows):
        assert total > 0 and bad == 0, f"case {case}: {bad} of {total} logits differ"
