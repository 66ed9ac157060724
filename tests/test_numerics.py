"""Numerics of libgs3d's own arithmetic helpers, checked on the CPU (no GPU): the same float
operations (IEEE binary32 with explicit fused multiply-adds) give the same bits on both."""
import subprocess
from pathlib import Path


REPO = Path(__file__).resolve().parent.parent

DIV_CHECK = r"""
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include "common.cuh"
using namespace gs3d;
static bool same(float a, float b) {
    if (a != a && b != b) return true;
    return std::memcmp(&a, &b, 4) == 0;
}
int main() {
    std::mt19937_64 rng(12345);
    std::uniform_real_distribution<double> e(-45.0, 39.0), m(1.0, 2.0);
    std::uniform_int_distribution<uint32_t> bits(0u, 0xffffffffu);
    long bad = 0, total = 0;
    auto draw = [&](int k) -> float {
        if (k % 11 == 0) { uint32_t u = bits(rng); float x; std::memcpy(&x, &u, 4); return x; }  // any pattern
        float x = (float)(m(rng) * std::pow(10.0, e(rng)));
        if (k % 13 == 0) x = std::ldexp(1.0f, -149 + (int)(bits(rng) % 60)) * (float)m(rng);  // subnormal..tiny
        if (k & 1) x = -x;
        if (k % 7 == 0) x = std::nextafter(x, 2 * x);
        return x;
    };
    const float specials[] = {0.0f, -0.0f, INFINITY, -INFINITY, NAN, 1e-45f, -1e-45f, 0x1p-100f,
                              0x1p-101f, 0x1p80f, 0x1p81f, 0x1p-60f, 0x1p-61f, 3.4e38f};
    // div_by_const: the bias corrections 1 - beta^t (and divisors outside the fast range)
    const float betas[4] = {0.9f, 0.999f, 0.5f, 0.99f};
    std::vector<float> bs;
    for (float beta : betas)
        for (int t = 1; t <= 40000; ++t) {
            const float b = 1.0f - (float)std::pow((double)beta, (double)t);
            if (t <= 200 || t % 97 == 0) bs.push_back(b);
        }
    for (float b : {0x1p-41f, 0x1p-40f, 1.5f, 0.0f, -0.25f}) bs.push_back(b);
    for (float b : bs) {
        const float rb = 1.0f / b;
        for (int k = 0; k < 3000; ++k) {
            const float x = draw(k);
            ++total; if (!same(div_by_const(x, b, rb), x / b)) ++bad;
        }
        for (float x : specials) { ++total; if (!same(div_by_const(x, b, rb), x / b)) ++bad; }
    }
    // div_small_num: numerators of every size over denominators sqrt(h) + eps and extremes
    for (int j = 0; j < 4000; ++j) {
        float d = (float)(m(rng) * std::pow(10.0, -15.0 + 20.0 * (j % 100) / 100.0));
        if (j % 50 == 0) d = specials[(j / 50) % 14];
        if (j % 77 == 0) d = -d;
        for (int k = 0; k < 2000; ++k) {
            const float x = draw(k);
            ++total; if (!same(div_small_num(x, d), x / d)) ++bad;
        }
        for (float x : specials) { ++total; if (!same(div_small_num(x, d), x / d)) ++bad; }
    }
    std::printf("%ld %ld\n", bad, total);
    return 0;
}
"""


def _build_and_run(tmp_path, name: str, source: str) -> tuple[int, int]:
    """Compile `source` (including csrc/common.cuh) as host code with nvcc and the library's
    floating-point flags; returns the program's (bad, total)."""
    import shutil
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    src = tmp_path / f"{name}.cu"
    src.write_text(source)
    exe = tmp_path / name
    csrc = REPO / "threedgaussiansplatting.jl_b200" / "csrc"
    subprocess.run([nvcc, "-std=c++17", "-O2", "-fmad=false", "-Xcompiler", "-ffp-contract=off",
                    f"-I{csrc}", str(src), "-o", str(exe)], check=True, capture_output=True)
    bad, total = map(int, subprocess.run([str(exe)], capture_output=True, text=True,
                                         check=True).stdout.split())
    return bad, total


def test_division_helpers_are_correctly_rounded(tmp_path):
    """div_by_const (Markstein quotient with the launch-constant reciprocal, exact detours for
    zero and tiny dividends) and div_small_num (zero and small numerators scaled) of
    csrc/common.cuh give the IEEE quotient bit for bit: normal, tiny, subnormal, zero, huge and
    non-finite operands, the Adam bias corrections and divisors outside the fast range."""
    bad, total = _build_and_run(tmp_path, "div", DIV_CHECK)
    assert total > 15_000_000
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
    bad, total = _build_and_run(tmp_path, "blend", BLEND_CHECK)
    assert total > 250_000_000
    assert bad == 0, f"{bad} of {total} results differ"


