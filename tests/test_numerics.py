"""Numerics of libgs3d's own arithmetic helpers, checked on the CPU (no GPU): the same float
operations (IEEE binary32 with explicit fused multiply-adds) give the same bits on both."""
import subprocess
import textwrap
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent

DIV_CHECK = r"""
#include <cmath>
#include <cstdio>
#include <cstdint>
#include <random>
#define GS_HD inline
static inline float fabsf_(float x) { return std::fabs(x); }
// the division helper of csrc/common.cuh, restated verbatim for the host
GS_HD float div_by_const(float x, float b, float rb) {
    const float ax = fabsf_(x);
    if (!(ax >= 1e-25f && ax <= 1e25f)) return x / b;
    const float q0 = x * rb;
    const float r = std::fmaf(-b, q0, x);
    return std::fmaf(r, rb, q0);
}
int main() {
    std::mt19937_64 rng(12345);
    std::uniform_real_distribution<double> e(-25.0, 25.0), m(1.0, 2.0);
    long bad = 0, total = 0;
    const float betas[4] = {0.9f, 0.999f, 0.5f, 0.99f};
    for (float beta : betas) {
        for (int t = 1; t <= 40000; ++t) {
            const float b = 1.0f - (float)std::pow((double)beta, (double)t);
            if (!(b > 0.0f)) continue;
            const float rb = 1.0f / b;
            const int n = t <= 200 ? 20000 : 200;
            for (int k = 0; k < n; ++k) {
                float x = (float)(m(rng) * std::pow(10.0, e(rng)));
                if (k & 1) x = -x;
                if (k % 7 == 0) x = std::nextafter(x, 2 * x);
                const float want = x / b, got = div_by_const(x, b, rb);
                ++total;
                if (std::memcmp(&want, &got, 4) != 0) ++bad;
            }
        }
    }
    std::printf("%ld %ld\n", bad, total);
    return 0;
}
"""


def test_division_by_launch_constant_is_correctly_rounded(tmp_path):
    src = tmp_path / "div.cpp"
    src.write_text("#include <cstring>\n" + DIV_CHECK)
    exe = tmp_path / "div"
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-mfma", str(src), "-o", str(exe)],
                   check=True)
    bad, total = map(int, subprocess.run([str(exe)], capture_output=True, text=True,
                                         check=True).stdout.split())
    assert total > 10_000_000
    assert bad == 0, f"{bad} of {total} quotients differ"


BLEND_CHECK = r"""
#include <cstdio>
#include <cstring>
#include "common.cuh"
using namespace gs3d;
static bool same(float a, float b) { return std::memcmp(&a, &b, 4) == 0; }
int main() {
    long bad = 0, total = 0;
    // every 7th float bit pattern of [-80, 0.5]
    const float lo = -80.0f, hi = 0.5f;
    uint32_t a, b;
    std::memcpy(&a, &hi, 4);
    for (uint32_t u = 0; u <= a; u += 7) {  // [0, 0.5]
        float x; std::memcpy(&x, &u, 4);
        ++total; if (!same(gs_expf_blend(x), gs_expf(x))) ++bad;
    }
    std::memcpy(&b, &lo, 4);
    for (uint32_t u = 0x80000000u; u <= b; u += 7) {  // [-80, -0]
        float x; std::memcpy(&x, &u, 4);
        ++total; if (!same(gs_expf_blend(x), gs_expf(x))) ++bad;
    }
    const float edge[] = {-80.0f, 0.5f, -80.00001f, 0.50001f, -88.0f, 88.0f, 100.0f, -200.0f,
                          1.0f, -1.0f, 0.0f, -0.0f};
    for (float x : edge) { ++total; if (!same(gs_expf_blend(x), gs_expf(x))) ++bad; }
    // min_hi(hi, x) == fmin_jl(hi, x) for non-NaN hi, over a spread of x
    const float his[] = {0.99f, 1.0f, 0.5f, 0.0f, 1e-30f};
    for (float h : his)
        for (uint32_t u = 0; u < 0xff800000u; u += 0x10001u) {
            float x; std::memcpy(&x, &u, 4);
            if (x != x) continue;
            ++total; if (!same(min_hi(h, x), fmin_jl(h, x))) ++bad;
        }
    std::printf("%ld %ld\n", bad, total);
    return 0;
}
"""


def test_blend_exp_fast_path_is_bit_identical(tmp_path):
    """The rasterisers' gs_expf_blend / min_hi (csrc/common.cuh, compiled here as host code by
    nvcc with the library's flags) against gs_expf / fmin_jl, bit for bit."""
    import shutil
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    src = tmp_path / "blend.cu"
    src.write_text(BLEND_CHECK)
    exe = tmp_path / "blend"
    csrc = REPO / "threedgaussiansplatting.jl_b200" / "csrc"
    subprocess.run([nvcc, "-std=c++17", "-O2", "-fmad=false", "-Xcompiler", "-ffp-contract=off",
                    f"-I{csrc}", str(src), "-o", str(exe)], check=True, capture_output=True)
    bad, total = map(int, subprocess.run([str(exe)], capture_output=True, text=True,
                                         check=True).stdout.split())
    assert total > 250_000_000
    assert bad == 0, f"{bad} of {total} results differ"


def test_division_helper_matches_library_source():
    """The restated helper above must stay identical to csrc/common.cuh's."""
    src = (REPO / "threedgaussiansplatting.jl_b200" / "csrc" / "common.cuh").read_text()
    for line in ("const float q0 = x * rb;", "const float r = fmaf(-b, q0, x);",
                 "return fmaf(r, rb, q0);", "if (!(ax >= 1e-25f && ax <= 1e25f)) return x / b;"):
        assert line in src
