/*
 * ORACLE — test infrastructure only.  Nothing in the product path may call
 * this file; it exists so tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg can check the CUDA path against a plain CPU restatement.
 *
 * Input generation, restated on the CPU:
 *
 *   include/random_fill.cuh:31-60 (fill_random) draws one value per element
 *   from std::mt19937(seed) through std::uniform_real_distribution<float>(lo,hi),
 *   narrows it to the device dtype with __float2bfloat16 (round to nearest
 *   even) and hands back the widened, post-rounding float as the host
 *   reference.  The reference is compiled by nvcc with gcc as host compiler,
 *   so the distribution is libstdc++'s:
 *     generate_canonical<float, 24>(g): one 32-bit draw u,
 *         r = (float)u / 2^32, clamped to nextafter(1, 0) when r rounds to 1;
 *     uniform_real_distribution: r * (hi - lo) + lo, in float.
 *   This file must be compiled with -ffp-contract=off (no FMA) so that the
 *   float arithmetic rounds exactly as the reference's host code does.
 *
 *   MT19937 itself is the published Matsumoto-Nishimura generator with the
 *   std::mt19937 parameters (w=32, n=624, m=397, r=31, a=0x9908b0df,
 *   u=11, s=7/b=0x9d2c5680, t=15/c=0xefc60000, l=18, f=1812433253).
 *
 * Parity pin: tests/test_oracle.py compares every function here against
 * fixtures produced by the reference's own fill_random (compiled from
 * include/random_fill.cuh by oracle/Makefile into oracle/_ref/) via
 * tests/golden/make_golden.py.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define MT_N 624
#define MT_M 397

typedef struct orc_mt19937 {
    uint32_t mt[MT_N];
    int idx;
} orc_mt19937;

void orc_mt_seed(orc_mt19937* g, uint32_t seed) {
    g->mt[0] = seed;
    for (int i = 1; i < MT_N; ++i) {
        uint32_t prev = g->mt[i - 1];
        g->mt[i] = 1812433253u * (prev ^ (prev >> 30)) + (uint32_t)i;
    }
    g->idx = MT_N;
}

static void mt_twist(orc_mt19937* g) {
    for (int i = 0; i < MT_N; ++i) {
        uint32_t y = (g->mt[i] & 0x80000000u) | (g->mt[(i + 1) % MT_N] & 0x7fffffffu);
        uint32_t v = g->mt[(i + MT_M) % MT_N] ^ (y >> 1);
        if (y & 1u) v ^= 0x9908b0dfu;
        g->mt[i] = v;
    }
    g->idx = 0;
}

uint32_t orc_mt_next(orc_mt19937* g) {
    if (g->idx >= MT_N) mt_twist(g);
    uint32_t y = g->mt[g->idx++];
    y ^= (y >> 11);
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= (y >> 18);
    return y;
}

/* libstdc++ generate_canonical<float, 24> over a 32-bit engine: one draw. */
static float canonical_f32(orc_mt19937* g) {
    const float sum = (float)orc_mt_next(g);
    const float scale = 4294967296.0f;
    float r = sum / scale;
    if (r >= 1.0f) r = nextafterf(1.0f, 0.0f);
    return r;
}

float orc_uniform_f32(orc_mt19937* g, float lo, float hi) {
    const float span = hi - lo;
    const float scaled = canonical_f32(g) * span;
    return scaled + lo;
}

/* __float2bfloat16 on the host: round to nearest even, NaN -> 0x7fff. */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)0x7fffu;
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/*
 * fill_random restated for a bf16 tensor of n elements.  `bits` receives the
 * bf16 payload that would be copied to the device, `ref` the widened floats
 * fill_random returns (either may be NULL).
 */
void orc_fill_random_bf16(uint32_t seed, float lo, float hi, size_t n,
                          uint16_t* bits, float* ref) {
    orc_mt19937 g;
    orc_mt_seed(&g, seed);
    for (size_t i = 0; i < n; ++i) {
        const float v = orc_uniform_f32(&g, lo, hi);
        const uint16_t b = orc_f32_to_bf16(v);
        if (bits) bits[i] = b;
        if (ref) ref[i] = orc_bf16_to_f32(b);
    }
}

/* fill_random for a float tensor: the pre-narrowing values themselves. */
void orc_fill_random_f32(uint32_t seed, float lo, float hi, size_t n, float* out) {
    orc_mt19937 g;
    orc_mt_seed(&g, seed);
    for (size_t i = 0; i < n; ++i) out[i] = orc_uniform_f32(&g, lo, hi);
}

/* --------------------------------------------------------------------------
 * OCP FP8 E4M3 (bias 7, no infinities, max finite 448, NaN = S.1111.111),
 * round to nearest even with saturation to +-448 — the arithmetic of the
 * PTX conversion cvt.rn.satfinite.e4m3x2.f32, restated from the format.
 * ------------------------------------------------------------------------ */
uint8_t orc_f32_to_e4m3(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint8_t)(sign | 0x7f);
    float a = fabsf(f);
    if (a >= 448.0f) return (uint8_t)(sign | 0x7e); /* satfinite */
    /* smallest subnormal is 2^-9; values are multiples of 2^-9 below 2^-6 */
    if (a < 0.015625f) { /* subnormal range: q = round(a / 2^-9) */
        float q = a * 512.0f;
        float fl = floorf(q);
        float rem = q - fl;
        uint32_t m = (uint32_t)fl;
        if (rem > 0.5f || (rem == 0.5f && (m & 1u))) m += 1u;
        /* m == 8 rounds up into the first normal binade (exp field 1, mant 0) */
        return (uint8_t)(sign | (uint8_t)m);
    }
    int e;
    float mant = frexpf(a, &e); /* a = mant * 2^e, mant in [0.5, 1) */
    /* a = 1.xxx * 2^(e-1): exponent field = e - 1 + 7 */
    int ef = e - 1 + 7;
    float scaled = mant * 16.0f; /* in [8, 16): 1.xxx scaled by 8 */
    float fl = floorf(scaled);
    float rem = scaled - fl;
    uint32_t m = (uint32_t)fl; /* 8..15 */
    if (rem > 0.5f || (rem == 0.5f && (m & 1u))) m += 1u;
    if (m == 16u) { m = 8u; ef += 1; }
    if (ef > 15 || (ef == 15 && m > 14u)) return (uint8_t)(sign | 0x7e);
    return (uint8_t)(sign | (uint8_t)(ef << 3) | (uint8_t)(m - 8u));
}

/* Per-row amax quantization (the fp8 workload's recipe): s[r] = amax_r / 448
   (1 for an all-zero row), q[r][c] = e4m3(x[r][c] / s[r]). */
void orc_quantize_e4m3_rows(const float* x, long rows, long cols, uint8_t* q, float* s) {
    for (long r = 0; r < rows; ++r) {
        const float* xr = x + r * cols;
        float amax = 0.0f;
        for (long c = 0; c < cols; ++c) {
            const float a = fabsf(xr[c]);
            if (a > amax) amax = a;
        }
        const float sc = amax > 0.0f ? amax / 448.0f : 1.0f;
        s[r] = sc;
        for (long c = 0; c < cols; ++c) q[r * cols + c] = orc_f32_to_e4m3(xr[c] / sc);
    }
}

float orc_e4m3_to_f32(uint8_t q) {
    const int sign = q & 0x80;
    const int ef = (q >> 3) & 0xf;
    const int m = q & 0x7;
    float v;
    if (ef == 0xf && m == 0x7) return NAN;
    if (ef == 0) v = ldexpf((float)m, -9);
    else v = ldexpf((float)(8 + m), ef - 10);
    return sign ? -v : v;
}
