// pi_oracle.cpp — CPU restatement of PowerInfer_x64's MoE feed-forward path
// and hot-neuron sparse FFN, used ONLY as a test/benchmark checker.
//
// TEST INFRASTRUCTURE. Nothing in the product library links or calls this
// file; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
// reference legs load it.
//
// The reference is Rust (no toolchain in this image), so this is a
// line-by-line C++ restatement of its CPU code. Every function cites the
// reference file:line it follows (paths relative to the reference project).
// Floating-point rules that make it match Rust bit for bit:
//   * built with -O2 -ffp-contract=off -fno-fast-math: Rust never fuses
//     a*b+c into an FMA;
//   * Rust f32::exp / f32::round map to libm expf / roundf (glibc here);
//   * the `half` crate (v2.4, Cargo.toml:20) converts f32->f16 with
//     round-to-nearest-even, restated in f32_to_f16 below;
//   * Rust `Iterator::sum` over f32 is a left fold (sequential adds).
//
// Parity pins: the reference's own known-answer tests for this path
// (src/quant/mod.rs:1263-1433, tests/smoke.rs:14-23, tests/soak.rs:68-85,
// src/moe/mod.rs:705-843, src/predictor/mod.rs:137-156) are restated as
// self-tests in tests/test_oracle.py. The Q8_0 int-dot numerics, the Q4_0
// matvec and MoE outputs have no golden vector in the reference: those are
// "parity unpinned" beyond the oracle's own cross-checks (SSE vs scalar
// bitwise, masked-dense identities, f64 bounds).

#include <cmath>
#include <cstdint>
#include <cstring>
#include <cstdlib>
#include <vector>
#include <thread>
#include <algorithm>
#include <numeric>
#include <mutex>
#include <smmintrin.h>
#include <pmmintrin.h>

extern "C" {

enum { QT_F32 = 0, QT_F16 = 1, QT_Q4_0 = 2, QT_Q8_0 = 8 };

// ---------------------------------------------------------------------------
// f16 <-> f32 (half crate 2.4 semantics: IEEE binary16, RNE, subnormals).
// ---------------------------------------------------------------------------
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: value = man * 2^-24
            float f = (float)man * 5.9604644775390625e-08f;
            std::memcpy(&bits, &f, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float out;
    std::memcpy(&out, &bits, 4);
    return out;
}

uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xff) {  // inf / nan (keep a quiet nan payload bit)
        if (man == 0) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | (man >> 13));
    }
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);  // overflow -> inf
    if (e <= 0) {
        // subnormal or zero in f16
        if (e < -10) return (uint16_t)sign;
        uint32_t m = man | 0x800000u;          // implicit bit
        int shift = 14 - e;                     // 14..24
        uint32_t half_man = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (half_man & 1u))) half_man++;
        return (uint16_t)(sign | half_man);
    }
    uint32_t half_man = man >> 13;
    uint32_t rem = man & 0x1fffu;
    uint32_t out = sign | ((uint32_t)e << 10) | half_man;
    if (rem > 0x1000u || (rem == 0x1000u && (half_man & 1u))) out++;  // may carry into exp: correct
    return (uint16_t)out;
}

static inline float ld_f16(const uint8_t* p) {
    uint16_t h = (uint16_t)p[0] | ((uint16_t)p[1] << 8);
    return or_f16_to_f32(h);
}
static inline float ld_f32(const uint8_t* p) {
    float f;
    std::memcpy(&f, p, 4);
    return f;
}

// ---------------------------------------------------------------------------
// Quantisers.
// ---------------------------------------------------------------------------

// Activation Q8_0 quantiser: src/quant/mod.rs:698-736 (quantize_f32_to_q8_0).
// Writes, per 32-block, the f16-rounded scale (as f32) and 32 int8 values.
// The reference pads a ragged final block with zeros (qs initialised to 0).
void or_quantize_act_q8_0(const float* x, int64_t n, float* scales, int8_t* qs) {
    int64_t nb = (n + 31) / 32;
    for (int64_t b = 0; b < nb; ++b) {
        int64_t base = b * 32, end = std::min<int64_t>(base + 32, n);
        float amax = 0.0f;
        for (int64_t i = base; i < end; ++i) {
            float a = std::fabs(x[i]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        scales[b] = or_f16_to_f32(or_f32_to_f16(d));
        int8_t* q = qs + b * 32;
        for (int i = 0; i < 32; ++i) q[i] = 0;
        for (int64_t i = base; i < end; ++i) {
            float v = x[i] * id;
            float r = std::round(v);  // Rust f32::round: half away from zero
            if (r != r) { q[i - base] = 0; continue; }  // `as i8` maps NaN to 0
            r = std::min(127.0f, std::max(-127.0f, r));
            q[i - base] = (int8_t)r;
        }
    }
}

// GGUF Q8_0 weight blocks (34 B: f16 d, 32 x i8) made with the same
// quantiser — the only Q8_0 quantiser in the reference (quant/mod.rs:698-736).
void or_quantize_q8_0(const float* x, int64_t n, uint8_t* out) {
    int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; ++b) {
        float sc;
        int8_t q[32];
        or_quantize_act_q8_0(x + b * 32, 32, &sc, q);
        // the stored f16 is f16(d); sc already equals f16_to_f32(f16(d)),
        // and f16(f16_to_f32(h)) == h, so re-encoding sc is exact.
        uint16_t h = or_f32_to_f16(sc);
        out[b * 34 + 0] = (uint8_t)(h & 0xff);
        out[b * 34 + 1] = (uint8_t)(h >> 8);
        std::memcpy(out + b * 34 + 2, q, 32);
    }
}

// GGUF Q4_0 weight blocks (18 B) with the quantiser BASELINE config 3 names:
// m = the value with the largest |x|, d = m / -8, id = 1/d, q = min(15,
// trunc(x*id + 8.5)). Nibbles are packed in the order the reference's
// decoder reads them (quant/mod.rs:193-199): byte i low nibble = element 2i,
// high nibble = element 2i+1, so dequantize_q4_0 inverts this packing.
void or_quantize_q4_0(const float* x, int64_t n, uint8_t* out) {
    int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; ++b) {
        const float* xb = x + b * 32;
        float amax = 0.0f, m = 0.0f;
        for (int i = 0; i < 32; ++i) {
            float a = std::fabs(xb[i]);
            if (a > amax) { amax = a; m = xb[i]; }
        }
        float d = m / -8.0f;
        float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        uint16_t h = or_f32_to_f16(d);
        uint8_t* o = out + b * 18;
        o[0] = (uint8_t)(h & 0xff);
        o[1] = (uint8_t)(h >> 8);
        for (int i = 0; i < 16; ++i) {
            float v0 = xb[2 * i] * id + 8.5f;
            float v1 = xb[2 * i + 1] * id + 8.5f;
            int q0 = (int)(int8_t)std::min(15.0f, std::max(-128.0f, std::trunc(v0)));
            int q1 = (int)(int8_t)std::min(15.0f, std::max(-128.0f, std::trunc(v1)));
            q0 = std::min(15, std::max(0, q0));
            q1 = std::min(15, std::max(0, q1));
            o[2 + i] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

// ---------------------------------------------------------------------------
// Dequantisation: quant/mod.rs:110-143 (dispatcher), :156-171 (F16),
// :180-204 (Q4_0, interleaved nibbles), :320-339 (Q8_0).
// Returns 0 on success, -1 when `len` is short (the reference's Err).
// ---------------------------------------------------------------------------
int or_dequantize(const uint8_t* data, int64_t len, int qtype, int64_t rows, int64_t cols, float* out) {
    int64_t n = rows * cols;
    if (qtype == QT_F32) {
        if (len < n * 4) return -1;
        for (int64_t i = 0; i < n; ++i) out[i] = ld_f32(data + 4 * i);
        return 0;
    }
    if (qtype == QT_F16) {
        if (len < n * 2) return -1;
        for (int64_t i = 0; i < n; ++i) out[i] = ld_f16(data + 2 * i);
        return 0;
    }
    int64_t bpr = cols / 32;
    int64_t nblk = rows * bpr;
    if (qtype == QT_Q4_0) {
        if (len < nblk * 18) return -1;
        for (int64_t b = 0; b < nblk; ++b) {
            const uint8_t* p = data + b * 18;
            float s = ld_f16(p);
            for (int i = 0; i < 16; ++i) {
                uint8_t byte = p[2 + i];
                out[b * 32 + 2 * i] = (float)((int)(byte & 0x0f) - 8) * s;
                out[b * 32 + 2 * i + 1] = (float)((int)((byte >> 4) & 0x0f) - 8) * s;
            }
        }
        return 0;
    }
    if (qtype == QT_Q8_0) {
        if (len < nblk * 34) return -1;
        for (int64_t b = 0; b < nblk; ++b) {
            const uint8_t* p = data + b * 34;
            float s = ld_f16(p);
            for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)(int8_t)p[2 + i] * s;
        }
        return 0;
    }
    return -2;
}

// ---------------------------------------------------------------------------
// Matvecs (GGML layout: W [ne0=n_in, ne1=n_out], one contiguous row per output).
// ---------------------------------------------------------------------------

// SSE4.1 block dot, restating matvec_q8_0_sse_range (quant/mod.rs:819-874).
__attribute__((target("sse4.1")))
static float q8_row_dot_sse(const uint8_t* row, const float* xs, const int8_t* xq, int64_t nblk) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 34;
        float ws = ld_f16(blk);
        const int8_t* wp = (const int8_t*)(blk + 2);
        const int8_t* xp = xq + b * 32;
        __m128i acc = _mm_setzero_si128();
        for (int k = 0; k < 32; k += 8) {
            __m128i w16 = _mm_cvtepi8_epi16(_mm_loadl_epi64((const __m128i*)(wp + k)));
            __m128i x16 = _mm_cvtepi8_epi16(_mm_loadl_epi64((const __m128i*)(xp + k)));
            acc = _mm_add_epi32(acc, _mm_madd_epi16(w16, x16));
        }
        __m128i hi = _mm_srli_si128(acc, 8);
        __m128i s2 = _mm_add_epi32(acc, hi);
        __m128i hi2 = _mm_srli_si128(s2, 4);
        int32_t sumi = _mm_cvtsi128_si32(_mm_add_epi32(s2, hi2));
        sumf += (float)sumi * (ws * xs[b]);
    }
    return sumf;
}

// Scalar block dot, restating matvec_q8_0_scalar (quant/mod.rs:877-899).
static float q8_row_dot_scalar(const uint8_t* row, const float* xs, const int8_t* xq, int64_t nblk) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < nblk; ++b) {
        const uint8_t* blk = row + b * 34;
        float ws = ld_f16(blk);
        int32_t sumi = 0;
        for (int i = 0; i < 32; ++i) sumi += (int32_t)(int8_t)blk[2 + i] * (int32_t)xq[b * 32 + i];
        sumf += (float)sumi * (ws * xs[b]);
    }
    return sumf;
}

static int g_use_scalar = 0;  // self-test hook: force the scalar restatement
void or_set_scalar(int on) { g_use_scalar = on; }

static inline float q8_row_dot(const uint8_t* row, const float* xs, const int8_t* xq, int64_t nblk) {
    return g_use_scalar ? q8_row_dot_scalar(row, xs, xq, nblk) : q8_row_dot_sse(row, xs, xq, nblk);
}

static int g_max_threads = 0;  // 0 = hardware_concurrency (num_cpus::get)
void or_set_threads(int n) { g_max_threads = n; }
static int ncpus() {
    int n = g_max_threads > 0 ? g_max_threads : (int)std::thread::hardware_concurrency();
    return n > 0 ? n : 1;
}

// matvec_col_major_q8_0: quant/mod.rs:652-689, threaded branch :741-810
// (rows split in ceil(n_out/n_threads) chunks when n_out >= 4096).
static void matvec_q8_0(float* y, const float* x, const uint8_t* raw, int64_t n_in, int64_t n_out) {
    int64_t nblk = n_in / 32;
    std::vector<float> xs(nblk);
    std::vector<int8_t> xq(nblk * 32);
    or_quantize_act_q8_0(x, n_in, xs.data(), xq.data());
    int64_t bpc = nblk * 34;
    int nt = ncpus();
    if (nt > 1 && n_out >= 4096) {
        int64_t chunk = (n_out + nt - 1) / nt;
        std::vector<std::thread> th;
        for (int c = 0; c < nt; ++c) {
            int64_t s = c * chunk;
            if (s >= n_out) break;
            int64_t e = std::min(n_out, s + chunk);
            th.emplace_back([=, &xs, &xq]() {
                for (int64_t j = s; j < e; ++j) y[j] = q8_row_dot(raw + j * bpc, xs.data(), xq.data(), nblk);
            });
        }
        for (auto& t : th) t.join();
        return;
    }
    for (int64_t j = 0; j < n_out; ++j) y[j] = q8_row_dot(raw + j * bpc, xs.data(), xq.data(), nblk);
}

// matvec_col_major_f32: quant/mod.rs:921-935.
static void matvec_f32(float* y, const float* x, const uint8_t* raw, int64_t n_in, int64_t n_out) {
    for (int64_t j = 0; j < n_out; ++j) {
        float sum = 0.0f;
        const uint8_t* r = raw + j * n_in * 4;
        for (int64_t i = 0; i < n_in; ++i) sum += ld_f32(r + 4 * i) * x[i];
        y[j] = sum;
    }
}

static int64_t raw_bytes(int qtype, int64_t n) {
    switch (qtype) {
        case QT_F32: return n * 4;
        case QT_F16: return n * 2;
        case QT_Q4_0: return n / 32 * 18;
        case QT_Q8_0: return n / 32 * 34;
    }
    return -1;
}

// matvec_col_major dispatcher: quant/mod.rs:939-970. Q8_0 -> int-dot path;
// F32 -> direct; anything else -> dequantise the whole matrix, then a
// sequential f32 dot (x[i] * w[j*n_in+i]).
int or_matvec_col_major(float* y, const float* x, const uint8_t* raw, int qtype, int64_t n_in, int64_t n_out) {
    if (qtype == QT_Q8_0 && n_in % 32 == 0) { matvec_q8_0(y, x, raw, n_in, n_out); return 0; }
    if (qtype == QT_F32) { matvec_f32(y, x, raw, n_in, n_out); return 0; }
    std::vector<float> w((size_t)(n_in * n_out));
    int rc = or_dequantize(raw, raw_bytes(qtype, n_in * n_out), qtype, 1, n_in * n_out, w.data());
    if (rc) return rc;
    for (int64_t j = 0; j < n_out; ++j) {
        float sum = 0.0f;
        for (int64_t i = 0; i < n_in; ++i) sum += x[i] * w[j * n_in + i];
        y[j] = sum;
    }
    return 0;
}

// matvec_col_major_select: quant/mod.rs:974-1068. Returns -3 on an
// out-of-range index (the reference's Err) — checked per index in order.
int or_matvec_col_major_select(float* y, const float* x, const uint8_t* raw, int qtype, int64_t n_in,
                               int64_t n_out, const int64_t* idx, int64_t n_idx) {
    if (n_idx == 0) return 0;
    if (qtype == QT_Q8_0 && n_in % 32 == 0) {
        int64_t nblk = n_in / 32, bpc = nblk * 34;
        std::vector<float> xs(nblk);
        std::vector<int8_t> xq(nblk * 32);
        or_quantize_act_q8_0(x, n_in, xs.data(), xq.data());
        for (int64_t s = 0; s < n_idx; ++s) {
            if (idx[s] < 0 || idx[s] >= n_out) return -3;
            y[s] = q8_row_dot_scalar(raw + idx[s] * bpc, xs.data(), xq.data(), nblk);
        }
        return 0;
    }
    if (qtype == QT_F32) {
        for (int64_t s = 0; s < n_idx; ++s) {
            if (idx[s] < 0 || idx[s] >= n_out) return -3;
            const uint8_t* r = raw + idx[s] * n_in * 4;
            float sum = 0.0f;
            for (int64_t i = 0; i < n_in; ++i) sum += x[i] * ld_f32(r + 4 * i);
            y[s] = sum;
        }
        return 0;
    }
    std::vector<float> w((size_t)(n_in * n_out));
    int rc = or_dequantize(raw, raw_bytes(qtype, n_in * n_out), qtype, 1, n_in * n_out, w.data());
    if (rc) return rc;
    for (int64_t s = 0; s < n_idx; ++s) {
        if (idx[s] < 0 || idx[s] >= n_out) return -3;
        float sum = 0.0f;
        for (int64_t i = 0; i < n_in; ++i) sum += x[i] * w[idx[s] * n_in + i];
        y[s] = sum;
    }
    return 0;
}

// matvec_col_major_sparse_input: quant/mod.rs:1073-1169. x holds the
// values at rows `idx`; y[c] = sum over (idx, x) pairs in the given order.
// Q8_0 uses f32 x against dequantised weights (x is NOT quantised here).
int or_matvec_col_major_sparse_input(float* y, const float* x, const int64_t* idx, int64_t n_idx,
                                     const uint8_t* raw, int qtype, int64_t n_in, int64_t n_out) {
    if (n_idx == 0) { for (int64_t c = 0; c < n_out; ++c) y[c] = 0.0f; return 0; }
    if (qtype == QT_Q8_0 && n_in % 32 == 0) {
        int64_t bpc = n_in / 32 * 34;
        for (int64_t c = 0; c < n_out; ++c) {
            float sum = 0.0f;
            for (int64_t s = 0; s < n_idx; ++s) {
                int64_t r = idx[s];
                if (r < 0 || r >= n_in) return -3;
                const uint8_t* blk = raw + c * bpc + (r / 32) * 34;
                float w = (float)(int8_t)blk[2 + r % 32] * ld_f16(blk);
                sum += x[s] * w;
            }
            y[c] = sum;
        }
        return 0;
    }
    if (qtype == QT_F32) {
        for (int64_t c = 0; c < n_out; ++c) {
            float sum = 0.0f;
            for (int64_t s = 0; s < n_idx; ++s) {
                int64_t r = idx[s];
                if (r < 0 || r >= n_in) return -3;
                sum += x[s] * ld_f32(raw + (c * n_in + r) * 4);
            }
            y[c] = sum;
        }
        return 0;
    }
    std::vector<float> w((size_t)(n_in * n_out));
    int rc = or_dequantize(raw, raw_bytes(qtype, n_in * n_out), qtype, 1, n_in * n_out, w.data());
    if (rc) return rc;
    for (int64_t c = 0; c < n_out; ++c) {
        float sum = 0.0f;
        for (int64_t s = 0; s < n_idx; ++s) {
            int64_t r = idx[s];
            if (r < 0 || r >= n_in) return -3;
            sum += x[s] * w[c * n_in + r];
        }
        y[c] = sum;
    }
    return 0;
}

// SiLU·up as quant/mod.rs:1196-1199: sig = 1/(1+exp(-g)); g = g*sig*up.
static inline float swiglu1(float g, float u) {
    float sig = 1.0f / (1.0f + std::exp(-g));
    return g * sig * u;
}

// ffn_swiglu_q: quant/mod.rs:1179-1204.
int or_ffn_swiglu_q(float* out, const float* x, const uint8_t* gate_raw, const uint8_t* up_raw,
                    const uint8_t* down_raw, int qtype, int64_t n_embd, int64_t n_ff) {
    std::vector<float> g(n_ff), u(n_ff);
    int rc = or_matvec_col_major(g.data(), x, gate_raw, qtype, n_embd, n_ff);
    if (!rc) rc = or_matvec_col_major(u.data(), x, up_raw, qtype, n_embd, n_ff);
    if (rc) return rc;
    for (int64_t i = 0; i < n_ff; ++i) g[i] = swiglu1(g[i], u[i]);
    return or_matvec_col_major(out, g.data(), down_raw, qtype, n_ff, n_embd);
}

// ffn_swiglu_q_selected: quant/mod.rs:1208-1249 (empty -> zeros;
// |S| >= n_ff -> dense ffn_swiglu_q).
int or_ffn_swiglu_q_selected(float* out, const float* x, const uint8_t* gate_raw, const uint8_t* up_raw,
                             const uint8_t* down_raw, int qtype, int64_t n_embd, int64_t n_ff,
                             const int64_t* idx, int64_t n_idx) {
    if (n_idx == 0) { for (int64_t c = 0; c < n_embd; ++c) out[c] = 0.0f; return 0; }
    if (n_idx >= n_ff) return or_ffn_swiglu_q(out, x, gate_raw, up_raw, down_raw, qtype, n_embd, n_ff);
    std::vector<float> g(n_idx), u(n_idx);
    int rc = or_matvec_col_major_select(g.data(), x, gate_raw, qtype, n_embd, n_ff, idx, n_idx);
    if (!rc) rc = or_matvec_col_major_select(u.data(), x, up_raw, qtype, n_embd, n_ff, idx, n_idx);
    if (rc) return rc;
    for (int64_t i = 0; i < n_idx; ++i) g[i] = swiglu1(g[i], u[i]);
    return or_matvec_col_major_sparse_input(out, g.data(), idx, n_idx, down_raw, qtype, n_ff, n_embd);
}

// ---------------------------------------------------------------------------
// RMSNorm with the reference's SSE lane order: ops.rs:13-27,
// simd.rs:116-137 (sum_squares_sse), :44-57 (hsum_sse), :139-172 (scale).
// ---------------------------------------------------------------------------
__attribute__((target("sse4.1")))
void or_rms_norm(float* out, const float* x, const float* w, int64_t n, float eps) {
    __m128 acc = _mm_setzero_ps();
    int64_t i = 0;
    for (; i + 4 <= n; i += 4) {
        __m128 v = _mm_loadu_ps(x + i);
        acc = _mm_add_ps(acc, _mm_mul_ps(v, v));
    }
    __m128 shuf = _mm_movehdup_ps(acc);
    __m128 sums = _mm_add_ps(acc, shuf);
    __m128 shuf2 = _mm_movehl_ps(sums, sums);
    float ss = _mm_cvtss_f32(_mm_add_ss(sums, shuf2));
    for (; i < n; ++i) ss += x[i] * x[i];
    float rms = std::sqrt(ss / (float)n + eps);
    float inv = 1.0f / rms;
    for (int64_t j = 0; j < n; ++j) out[j] = x[j] * inv;
    for (int64_t j = 0; j < n; ++j) out[j] *= w[j];
}

// ---------------------------------------------------------------------------
// MoE routing: model/mod.rs:1254-1312.
//   logits = matvec_col_major(F32 router [ne0=d, ne1=E])   (:1262-1270)
//   probs = softmax (exp(l - max) / sequential sum)        (:1279-1283)
//   top-k by probs; the reference's select_nth_unstable_by leaves the order
//   of equal probabilities unspecified — this restatement breaks ties to the
//   lowest expert index               (:1286-1292)
//   selected indices sorted ascending                      (:1303)
//   gates = probs[sel] / sequential sum (if sum > 0)       (:1306-1312)
// An optional per-expert logit bias (BASELINE config 3's Zipf skew; not in
// the reference) is added to the logits before the softmax.
// Dispatch outputs (no counterpart in the reference, which loops token by
// token): counts[e], offsets = exclusive prefix sum, perm[offsets[e]+r] =
// the r-th token (ascending) routed to e.
// ---------------------------------------------------------------------------
static void route_one(const float* x, const uint8_t* router, const float* bias, int64_t d, int E, int k,
                      float* logits_out, int32_t* idx, float* gates) {
    std::vector<float> logits(E);
    matvec_f32(logits.data(), x, router, d, E);
    if (bias) for (int e = 0; e < E; ++e) logits[e] = logits[e] + bias[e];
    if (logits_out) std::memcpy(logits_out, logits.data(), sizeof(float) * E);
    float mx = -INFINITY;
    for (int e = 0; e < E; ++e) mx = std::fmax(mx, logits[e]);
    std::vector<float> ex(E), probs(E);
    for (int e = 0; e < E; ++e) ex[e] = std::exp(logits[e] - mx);
    float es = 0.0f;
    for (int e = 0; e < E; ++e) es += ex[e];
    for (int e = 0; e < E; ++e) probs[e] = ex[e] / es;
    std::vector<int> order(E);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return probs[a] > probs[b]; });
    std::vector<int> sel(order.begin(), order.begin() + k);
    std::sort(sel.begin(), sel.end());
    float ssum = 0.0f;
    for (int j = 0; j < k; ++j) ssum += probs[sel[j]];
    for (int j = 0; j < k; ++j) {
        idx[j] = sel[j];
        gates[j] = ssum > 0.0f ? probs[sel[j]] / ssum : probs[sel[j]];
    }
}

// Runs fn(t0, t1) over token ranges on `threads` host threads (0 = all cores).
// Tokens are independent in the reference's loop (model/mod.rs:1234), so the
// split changes no result; it only lets the checker keep up with GPU-sized batches.
}  // extern "C"
template <typename F>
static void over_tokens(int64_t T, int threads, F fn) {
    int n = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
    if (n <= 1 || T < 2) { fn(0, T); return; }
    n = (int)std::min<int64_t>(n, T);
    std::vector<std::thread> pool;
    for (int i = 0; i < n; ++i) {
        const int64_t t0 = T * i / n, t1 = T * (i + 1) / n;
        pool.emplace_back([=] { fn(t0, t1); });
    }
    for (auto& th : pool) th.join();
}
extern "C" {

void or_moe_route_mt(const float* x, int64_t T, const uint8_t* router, const float* bias, int64_t d, int E, int k,
                     float* logits, int32_t* idx, float* gates, int32_t* counts, int32_t* offsets, int32_t* perm,
                     int threads) {
    over_tokens(T, threads, [&](int64_t t0, int64_t t1) {
        for (int64_t t = t0; t < t1; ++t)
            route_one(x + t * d, router, bias, d, E, k, logits ? logits + t * E : nullptr, idx + t * k, gates + t * k);
    });
    if (!counts) return;
    for (int e = 0; e < E; ++e) counts[e] = 0;
    for (int64_t t = 0; t < T * k; ++t) counts[idx[t]]++;
    int32_t run = 0;
    for (int e = 0; e < E; ++e) { offsets[e] = run; run += counts[e]; }
    if (!perm) return;
    std::vector<int32_t> fill(offsets, offsets + E);
    for (int64_t t = 0; t < T; ++t)
        for (int j = 0; j < k; ++j) perm[fill[idx[t * k + j]]++] = (int32_t)t;
}

void or_moe_route(const float* x, int64_t T, const uint8_t* router, const float* bias, int64_t d, int E, int k,
                  float* logits, int32_t* idx, float* gates, int32_t* counts, int32_t* offsets, int32_t* perm) {
    or_moe_route_mt(x, T, router, bias, d, E, k, logits, idx, gates, counts, offsets, perm, 1);
}

// MoeRouter::route of the standalone operator API (moe/mod.rs:69-108) for T tokens:
//   logits[j] = sum_i x[i] * gate[i*E + j], sequential in i (ops::matvec_t, ops.rs:251-259);
//   the top_k largest logits (select_nth_unstable_by leaves equal logits in an
//   unspecified order: this restatement keeps the lowest index), ordered by
//   descending logit (a stable sort: equal logits stay in ascending index order);
//   weights = ops::softmax of the selected logits (ops.rs:160-180: max, v = exp(v - max)
//   with a sequential sum, then v *= 1/sum).
// gate: row-major [d][E]; idx/weights: [T][k] in the reference's output order.
void or_moe_api_route(const float* x, int64_t T, const float* gate, int64_t d, int E, int k, int32_t* idx,
                      float* weights, int threads) {
    over_tokens(T, threads, [&](int64_t t0, int64_t t1) {
        std::vector<float> logits(E);
        std::vector<int> order(E);
        for (int64_t t = t0; t < t1; ++t) {
            const float* xt = x + t * d;
            for (int j = 0; j < E; ++j) {
                float sum = 0.0f;
                for (int64_t i = 0; i < d; ++i) sum += xt[i] * gate[i * E + j];
                logits[j] = sum;
            }
            std::iota(order.begin(), order.end(), 0);
            std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return logits[a] > logits[b]; });
            float mx = -INFINITY;
            for (int j = 0; j < k; ++j) mx = std::fmax(mx, logits[order[j]]);
            std::vector<float> w(k);
            float sum = 0.0f;
            for (int j = 0; j < k; ++j) {
                w[j] = std::exp(logits[order[j]] - mx);
                sum += w[j];
            }
            const float inv = 1.0f / sum;
            for (int j = 0; j < k; ++j) {
                idx[t * k + j] = order[j];
                weights[t * k + j] = w[j] * inv;
            }
        }
    });
}

// ---------------------------------------------------------------------------
// Full MoE layer, one token at a time: model/mod.rs:1245-1571 (the path
// that runs when no hot-expert cache is set), followed optionally by the
// residual add (:1627-1633) and preceded optionally by RMSNorm (:1239).
//   gate_exps / up_exps: [ne0=d, ne1=f, ne2=E]; down_exps: [ne0=f, ne1=d, ne2=E]
//   expert e's bytes = [e*B, (e+1)*B), B = ceil(ne0*ne1/32)*block_bytes
//   (weights.rs:78-113).
// Experts run on 2 threads (first k/2, rest) and the shared expert on the
// calling thread when cores >= 3 (:1430-1537), else after the join
// (:1541-1570); combine: ascending expert index, then the shared expert.
// threads: 0 -> restate the reference's threading; 1 -> single thread.
// ---------------------------------------------------------------------------
struct OrMoeLayer {
    int64_t d, f, f_sh;
    int E, k, qtype;
    const uint8_t* router;     // f32 [d x E]
    const float* bias;         // [E] or null
    const uint8_t* gate_exps;
    const uint8_t* up_exps;
    const uint8_t* down_exps;
    const uint8_t* gate_sh;    // null = no shared expert
    const uint8_t* up_sh;
    const uint8_t* down_sh;
    const float* shared_gate;  // [d] or null (scale 1)
};

int or_moe_layer(const OrMoeLayer* L, const float* x_in, int64_t T, float* out, int threads, int residual,
                 int rmsnorm, float eps) {
    int64_t d = L->d, f = L->f;
    int64_t B_gu = raw_bytes(L->qtype, d * f), B_d = raw_bytes(L->qtype, f * d);
    int cores = threads == 1 ? 1 : ncpus();
    std::vector<float> normed(d), ffn(d), ones(d, 1.0f);
    std::vector<int32_t> idx(L->k);
    std::vector<float> gates(L->k);
    for (int64_t t = 0; t < T; ++t) {
        const float* x = x_in + t * d;
        if (rmsnorm) or_rms_norm(normed.data(), x, ones.data(), d, eps);
        else std::memcpy(normed.data(), x, sizeof(float) * d);
        route_one(normed.data(), L->router, L->bias, d, L->E, L->k, nullptr, idx.data(), gates.data());
        std::fill(ffn.begin(), ffn.end(), 0.0f);
        int k = L->k, mid = k / 2;
        std::vector<std::vector<float>> eo(k, std::vector<float>(d));
        int rc1 = 0, rc2 = 0, rcs = 0;
        auto run = [&](int lo, int hi, int* rc) {
            for (int j = lo; j < hi && !*rc; ++j) {
                int e = idx[j];
                *rc = or_ffn_swiglu_q(eo[j].data(), normed.data(), L->gate_exps + e * B_gu, L->up_exps + e * B_gu,
                                      L->down_exps + e * B_d, L->qtype, d, f);
            }
        };
        std::vector<float> sh(d);
        float scale = 1.0f;
        auto shared = [&]() {
            if (!L->gate_sh) return;
            rcs = or_ffn_swiglu_q(sh.data(), normed.data(), L->gate_sh, L->up_sh, L->down_sh, L->qtype, d, L->f_sh);
            if (L->shared_gate) {
                float dot = 0.0f;
                for (int64_t i = 0; i < d; ++i) dot += L->shared_gate[i] * normed[i];
                scale = 1.0f / (1.0f + std::exp(-dot));
            }
        };
        if (threads == 1) {
            run(0, k, &rc1);
            shared();
        } else {
            std::thread t1([&] { run(0, mid, &rc1); });
            std::thread t2([&] { run(mid, k, &rc2); });
            if (cores >= 3) shared();
            t1.join();
            t2.join();
            if (cores < 3) shared();
        }
        if (rc1 || rc2 || rcs) return rc1 ? rc1 : (rc2 ? rc2 : rcs);
        for (int j = 0; j < k; ++j)
            for (int64_t c = 0; c < d; ++c) ffn[c] += gates[j] * eo[j][c];
        if (L->gate_sh)
            for (int64_t c = 0; c < d; ++c) ffn[c] += scale * sh[c];
        float* o = out + t * d;
        if (residual) for (int64_t c = 0; c < d; ++c) o[c] = x[c] + ffn[c];
        else std::memcpy(o, ffn.data(), sizeof(float) * d);
    }
    return 0;
}

// The same layer for a batch of independent tokens spread over host threads
// (each token runs the single-threaded path, so the outputs equal or_moe_layer's).
int or_moe_layer_mt(const OrMoeLayer* L, const float* x_in, int64_t T, float* out, int residual, int rmsnorm,
                    float eps, int threads) {
    int rc = 0;
    std::mutex mu;
    over_tokens(T, threads, [&](int64_t t0, int64_t t1) {
        int r = or_moe_layer(L, x_in + t0 * L->d, t1 - t0, out + t0 * L->d, 1, residual, rmsnorm, eps);
        if (r) { std::lock_guard<std::mutex> g(mu); rc = r; }
    });
    return rc;
}

// Hot-neuron sparse dense FFN for a batch of tokens, each with its own
// ascending index list (CSR: idx[ptr[t] .. ptr[t+1])): the per-token call of
// ffn_swiglu_q_selected at model/mod.rs:1601-1612.
int or_sparse_ffn(const float* x, int64_t T, const uint8_t* gate_raw, const uint8_t* up_raw, const uint8_t* down_raw,
                  int qtype, int64_t n_embd, int64_t n_ff, const int64_t* ptr, const int64_t* idx, float* out) {
    for (int64_t t = 0; t < T; ++t) {
        int rc = or_ffn_swiglu_q_selected(out + t * n_embd, x + t * n_embd, gate_raw, up_raw, down_raw, qtype, n_embd,
                                          n_ff, idx + ptr[t], ptr[t + 1] - ptr[t]);
        if (rc) return rc;
    }
    return 0;
}

// ---------------------------------------------------------------------------
// Host generator of the benchmark's synthetic inputs (no reference counterpart:
// the reference publishes no data for this path). Value i of a stream is a
// Box-Muller normal from SplitMix64 outputs 2*(i/2) and 2*(i/2)+1
// (SplitMix64 as model/mod.rs:2041-2061), cos for even i, sin for odd i,
// scaled by stdv. It lets the CPU legs build their inputs without the GPU
// library.
// ---------------------------------------------------------------------------
static inline uint64_t sm64_at(uint64_t seed, uint64_t j) {
    uint64_t z = seed + (j + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline float synth_one(uint64_t seed, uint64_t i, float stdv) {
    const uint64_t m = i >> 1;
    const double u1 = 1.0 - (double)(sm64_at(seed, 2 * m) >> 11) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(sm64_at(seed, 2 * m + 1) >> 11) * (1.0 / 9007199254740992.0);
    const double r = std::sqrt(-2.0 * std::log(u1));
    const double th = 6.283185307179586 * u2;
    const double v = (i & 1) ? r * std::sin(th) : r * std::cos(th);
    return (float)(v * (double)stdv);
}

void or_synth_normal(uint64_t seed, uint64_t offset, int64_t n, float stdv, float* out, int threads) {
    over_tokens(n, threads, [&](int64_t a, int64_t b) {
        for (int64_t k = a; k < b; ++k) out[k] = synth_one(seed, offset + (uint64_t)k, stdv);
    });
}

// n_mats [rows x cols] matrices ~ N(0, stdv) from one stream, quantised with this
// file's Q8_0 (qtype 8) or Q4_0 (qtype 2) weight quantiser into GGUF bytes.
void or_synth_quant(uint64_t seed, int64_t n_mats, int64_t rows, int64_t cols, int qtype, float stdv, uint8_t* out,
                    int threads) {
    const int64_t n = n_mats * rows * cols, nblk = n / 32, bb = qtype == QT_Q8_0 ? 34 : 18;
    over_tokens(nblk, threads, [&](int64_t b0, int64_t b1) {
        float buf[32];
        for (int64_t b = b0; b < b1; ++b) {
            for (int i = 0; i < 32; ++i) buf[i] = synth_one(seed, (uint64_t)(b * 32 + i), stdv);
            if (qtype == QT_Q8_0) or_quantize_q8_0(buf, 32, out + b * bb);
            else or_quantize_q4_0(buf, 32, out + b * bb);
        }
    });
}

// Predictor::predict / predict_hot: predictor/mod.rs:63-95 (ndarray dot is
// a sequential sum per output row here). W1 [hidden x in], W2 [out x hidden].
void or_predictor(const float* a, const float* W1, const float* b1, const float* W2, const float* b2, int64_t n_in,
                  int64_t n_hidden, int64_t n_out, float* probs) {
    std::vector<float> h(n_hidden);
    for (int64_t j = 0; j < n_hidden; ++j) {
        float s = 0.0f;
        for (int64_t i = 0; i < n_in; ++i) s += W1[j * n_in + i] * a[i];
        s = s + b1[j];
        h[j] = std::fmax(s, 0.0f);
    }
    for (int64_t j = 0; j < n_out; ++j) {
        float s = 0.0f;
        for (int64_t i = 0; i < n_hidden; ++i) s += W2[j * n_hidden + i] * h[i];
        s = s + b2[j];
        probs[j] = 1.0f / (1.0f + std::exp(-s));
    }
}

}  // extern "C"
