// oracle_math.h — TEST INFRASTRUCTURE ONLY (the CPU oracle of gs3d). Nothing in the
// product (the gs3d package, libgs3d.so) may include, link or call anything under oracle/.
//
// Scalar primitives of the CPU restatement of ThreeDGaussianSplatting.jl's GPU path.
// Transcendentals are defined here from published methods (not taken from any libm), so
// that the CUDA build, which implements the same methods independently, can be compared
// bit for bit:
//   * exp: Cody & Waite argument reduction x = k ln2 + r, |r| <= ln2/2 (W. J. Cody and
//     W. Waite, "Software Manual for the Elementary Functions", 1980), then the degree-7
//     Taylor polynomial of e^r in Horner form with fused multiply-adds, scaled by 2^k.
//   * log: x = 2^e m with m in [sqrt(1/2), sqrt(2)), log m = 2 atanh(s), s = (m-1)/(m+1),
//     atanh by its odd Taylor series through s^9 (|s| <= 0.1716).
// Both are accurate to about 1-2 ulp; tests/test_oracle_golden.py checks them against libm.
// Compile with -ffp-contract=off: every a*b+c below is two roundings unless written fmaf.
#pragma once
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <climits>
#include <thread>
#include <vector>

namespace oracle {

// Host threads used by the loops whose iterations are independent (per Gaussian, per tile).
// Results do not depend on the thread count except for the order of the backward pass's
// double-precision sums.
inline int& thread_count() { static int n = 1; return n; }

template <class Fn>
void parallel_for(int64_t begin, int64_t end, Fn fn) {
    const int nt = thread_count();
    if (nt <= 1 || end - begin < 64) {
        for (int64_t i = begin; i < end; ++i) fn(i);
        return;
    }
    std::atomic<int64_t> next(begin);
    const int64_t chunk = std::max<int64_t>(1, (end - begin) / ((int64_t)nt * 32));
    auto worker = [&]() {
        for (;;) {
            const int64_t s = next.fetch_add(chunk);
            if (s >= end) break;
            const int64_t e = std::min(end, s + chunk);
            for (int64_t i = s; i < e; ++i) fn(i);
        }
    };
    std::vector<std::thread> th;
    for (int t = 1; t < nt; ++t) th.emplace_back(worker);
    worker();
    for (auto& t : th) t.join();
}

// a += v on a double shared between threads
inline void atomic_add(double* a, double v) {
    uint64_t old = __atomic_load_n(reinterpret_cast<uint64_t*>(a), __ATOMIC_RELAXED);
    for (;;) {
        double cur;
        std::memcpy(&cur, &old, 8);
        const double nv = cur + v;
        uint64_t nb;
        std::memcpy(&nb, &nv, 8);
        if (__atomic_compare_exchange_n(reinterpret_cast<uint64_t*>(a), &old, nb, true,
                                        __ATOMIC_RELAXED, __ATOMIC_RELAXED))
            return;
    }
}

static inline float bits_to_float(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
static inline uint32_t float_to_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

static inline float o_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    const float k = std::rint(x * 1.44269502162933349609375f);  // x / ln2, ties to even
    float r = std::fmaf(-k, 0.693147182464599609375f, x);       // ln2 rounded to float
    r = std::fmaf(-k, -1.904654323148236e-09f, r);              // ln2 - float(ln2)
    float p = 1.98412698e-04f;                                  // 1/5040
    p = std::fmaf(p, r, 1.38888892e-03f);                       // 1/720
    p = std::fmaf(p, r, 8.33333377e-03f);                       // 1/120
    p = std::fmaf(p, r, 4.16666679e-02f);                       // 1/24
    p = std::fmaf(p, r, 1.66666672e-01f);                       // 1/6
    p = std::fmaf(p, r, 0.5f);
    p = std::fmaf(p, r, 1.0f);
    p = std::fmaf(p, r, 1.0f);
    // p * 2^k in two exact power-of-two steps (k in [-151, 128])
    const int ki = (int)k;
    const int k1 = ki / 2;
    const int k2 = ki - k1;
    const float s1 = bits_to_float((uint32_t)(k1 + 127) << 23);
    const float s2 = bits_to_float((uint32_t)(k2 + 127) << 23);
    return (p * s1) * s2;
}

static inline float o_logf(float x) {
    if (x != x) return x;
    if (x < 0.0f) return NAN;
    if (x == 0.0f) return -INFINITY;
    if (x == INFINITY) return INFINITY;
    int e_adj = 0;
    if (x < 1.17549435e-38f) { x = x * 8388608.0f; e_adj = -23; }  // 2^23, exact
    const uint32_t u = float_to_bits(x);
    int e = (int)((u >> 23) & 0xffu) - 127 + e_adj;
    float m = bits_to_float((u & 0x007fffffu) | 0x3f800000u);         // [1, 2)
    if (m > 1.41421353816986083984375f) { m = m * 0.5f; e += 1; }      // [0.7071, 1.4142]
    const float f = m - 1.0f;                                          // exact (Sterbenz)
    const float s = f / (2.0f + f);
    const float s2 = s * s;
    float p = std::fmaf(s2, 0.111111112f, 0.142857149f);               // 1/9, 1/7
    p = std::fmaf(p, s2, 0.2f);                                        // 1/5
    p = std::fmaf(p, s2, 0.333333343f);                                // 1/3
    const float t = (s * s2) * p;
    const float logm = 2.0f * s + 2.0f * t;
    const float ef = (float)e;
    return std::fmaf(ef, 0.693147182464599609375f, std::fmaf(ef, -1.904654323148236e-09f, logm));
}

// sigmoid(x) = 1 / (1 + exp(-x))  (misc.jl:185-187)
static inline float o_sigmoid(float x) { return 1.0f / (1.0f + o_expf(-x)); }
// logit(x) = -log(1/x - 1)  (misc.jl:194-196)
static inline float o_logit(float x) { return -o_logf(1.0f / x - 1.0f); }

// Julia clamp(x, lo, hi) = x > hi ? hi : (x < lo ? lo : x)
// Julia min(a, b) for floats: NaN if either argument is NaN
static inline float o_min(float a, float b) { return (a != a || b != b) ? a + b : (b < a ? b : a); }

static inline float o_clamp(float x, float lo, float hi) { return x > hi ? hi : (x < lo ? lo : x); }

// Float -> Int32 with saturation; NaN -> 0 (the reference would throw InexactError; this
// build defines NaN/overflowing bounding boxes as empty, identically on CPU and GPU).
static inline int32_t o_sat_i32(float v) {
    if (v != v) return 0;
    if (v >= 2147483520.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int32_t)v;
}
static inline int32_t o_ceil_i32(float v) { return o_sat_i32(std::ceil(v)); }
static inline int32_t o_round_i32(float v) { return o_sat_i32(std::rint(v)); }  // ties to even

// SH constants (sh.jl:1-18), rounded to Float32 like F(SH_CONSTS_F64[i]).
static const float SH_C[16] = {
    (float)0.28209479177387814, (float)0.4886025119029199, (float)0.4886025119029199,
    (float)0.4886025119029199, (float)1.0925484305920792, (float)-1.0925484305920792,
    (float)0.31539156525252005, (float)-1.0925484305920792, (float)0.5462742152960396,
    (float)-0.5900435899266435, (float)2.890611442640554, (float)-0.4570457994644658,
    (float)0.3731763325901154, (float)-0.4570457994644658, (float)1.445305721320277,
    (float)-0.5900435899266435};

// evaluate_sh_basis_function(i, direction) (sh.jl:123-149), i 1-based.
static inline float o_sh_basis(int i, float x, float y, float z) {
    switch (i) {
        case 1: return SH_C[0];
        case 2: return -y * SH_C[1];
        case 3: return z * SH_C[2];
        case 4: return -x * SH_C[3];
        case 5: return x * y * SH_C[4];
        case 6: return y * z * SH_C[5];
        case 7: return (2.0f * (z * z) - x * x - y * y) * SH_C[6];
        case 8: return x * z * SH_C[7];
        case 9: return (x * x - y * y) * SH_C[8];
        case 10: return y * (3.0f * (x * x) - y * y) * SH_C[9];
        case 11: return x * y * z * SH_C[10];
        case 12: return y * (4.0f * (z * z) - x * x - y * y) * SH_C[11];
        case 13: return z * (2.0f * (z * z) - 3.0f * (x * x + y * y)) * SH_C[12];
        case 14: return x * (4.0f * (z * z) - x * x - y * y) * SH_C[13];
        case 15: return z * (x * x - y * y) * SH_C[14];
        case 16: return x * (x * x - 3.0f * (y * y)) * SH_C[15];
        default: return 0.0f;
    }
}

}  // namespace oracle
