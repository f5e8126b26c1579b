"""The exact-order helpers of the device code (katgpt-rs_b200/csrc/kg_exact.cuh:
simd_dot_f32 at compile-time and run-time lengths, simd_sum_sq, simd_sum_f32
at run-time lengths, the Cephes exp lanes with and without the clamp and its
scalar tail, and the LoRA update lora_apply16) compiled as plain C++ and held
against the oracle's restatements bit for bit, on the CPU: the same source the
exact micro kernels use, so their arithmetic is checked without a GPU."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

DRIVER = r"""
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>
#include "kg_exact.cuh"
extern "C" {
float or_dot(const float *a, const float *b, int64_t n);
float or_sum_sq(const float *x, int64_t n);
float or_sum(const float *x, int64_t n);
void or_exp_inplace(float *x, int64_t n);
float or_exp_sum_inplace(float *x, int64_t n);
float or_scalar_exp(float x);
void or_lora_apply(int64_t rank, int64_t in_dim, int64_t out_dim, float alpha, const float *a, const float *b,
                   const float *in, float *out);
}
static long bad = 0, total = 0;
static void same(float a, float b) { ++total; if (std::memcmp(&a, &b, 4)) ++bad; }
template <int LEN> static void check_len(std::mt19937 &g) {
    std::normal_distribution<float> nd(0.f, 1.f);
    for (int t = 0; t < 200; ++t) {
        float a[LEN], b[LEN];
        for (int i = 0; i < LEN; ++i) a[i] = nd(g), b[i] = nd(g);
        same(kgx::dot<LEN>(a, b), or_dot(a, b, LEN));
        same(kgx::sum_sq<LEN>(a), or_sum_sq(a, LEN));
    }
}
int main() {
    std::mt19937 g(7);
    std::normal_distribution<float> nd(0.f, 1.f);
    check_len<4>(g); check_len<16>(g); check_len<24>(g); check_len<40>(g); check_len<64>(g);
    check_len<100>(g); check_len<768>(g);
    for (int t = 0; t < 2000; ++t) {
        const int len = 1 + t % 16;
        float a[16], b[16];
        for (int i = 0; i < 16; ++i) a[i] = nd(g), b[i] = nd(g);
        same(kgx::dot_rt16(a, b, len), or_dot(a, b, len));
    }
    // Cephes exp: vector lanes with the clamp (simd_exp_inplace), without it
    // (the exp_sum variant), and the scalar tail; sums over run-time lengths
    std::uniform_real_distribution<float> wide(-110.0f, 95.0f);
    for (int t = 0; t < 4000; ++t) {
        float v[8], e[8], f[8];
        for (int l = 0; l < 8; ++l) v[l] = e[l] = f[l] = t % 2 ? wide(g) : nd(g) * 8.0f;
        or_exp_inplace(e, 8);
        or_exp_sum_inplace(f, 8);
        for (int l = 0; l < 8; ++l) {
            same(kgx::cephes_lane(v[l], true), e[l]);
            same(kgx::cephes_lane(v[l], false), f[l]);
            same(kgx::cephes_scalar(v[l]), or_scalar_exp(v[l]));
        }
    }
    for (int t = 0; t < 3000; ++t) {
        const int n = 1 + t % 64;
        float x[64];
        for (int i = 0; i < 64; ++i) x[i] = nd(g);
        same(kgx::sum_rt<64>(x, n), or_sum(x, n));
        if (n < 32) same(kgx::sum_small<31>(x, n), or_sum(x, n));
    }
    for (int t = 0; t < 5000; ++t) {
        const int rank = 1 + g() % 16, in_dim = 1 + g() % 16, out_dim = 1 + g() % 16;
        const float alpha = t % 3 == 0 ? 8.0f : nd(g) * 4.0f;
        std::vector<float> A(rank * in_dim), B(out_dim * rank);
        for (auto &v : A) v = nd(g);
        for (auto &v : B) v = nd(g);
        float in[64], out[64], ref[64];
        for (auto &v : in) v = nd(g);
        for (int i = 0; i < 64; ++i) out[i] = ref[i] = nd(g);
        kgx::lora_apply16(out, in, A.data(), B.data(), rank, in_dim, out_dim, alpha / (float)rank);
        or_lora_apply(rank, in_dim, out_dim, alpha, A.data(), B.data(), in, ref);
        for (int i = 0; i < 64; ++i) same(out[i], ref[i]);
    }
    std::printf("%ld %ld\n", bad, total);
    return 0;
}
"""


def test_exact_helpers_match_the_oracle(orc, tmp_path):
    lib = orc.lib()                                   # builds oracle/_build/libkgoracle.so if needed
    libdir = os.path.dirname(lib._name)
    src = tmp_path / "exact_host.cpp"
    src.write_text(DRIVER)
    exe = tmp_path / "exact_host"
    cmd = ["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math",
           "-I", os.path.join(ROOT, "katgpt-rs_b200", "csrc"), str(src), "-L", libdir, "-lkgoracle",
           "-Wl,-rpath," + libdir, "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        pytest.fail(r.stderr[-2000:])
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    bad, total = int(out[0]), int(out[1])
    assert total > 300000 and bad == 0, f"{bad} of {total} differ"
