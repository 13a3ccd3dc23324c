// Per-function drop-ins for the reference's quant:: operators on raw GGUF
// bytes, the hot-neuron sparse FFN, the predictor MLP, weight quantisers and
// the synthetic-input generator.
//
// The per-function drop-ins (pi_matvec_col_major & co.) read the GGUF
// array-of-blocks bytes in place and keep the reference's summation order
// exactly (one sequential f32 chain per output, mul then add, no FMA), so
// they are bit-identical to the reference whenever its exp rounding agrees.
// The sparse-FFN object instead repacks its weights and parallelises the
// sums (results within the stated tolerance).
#include "pi_common.cuh"
#include "pi_internal.h"

#include <cmath>

namespace {

// --------------------------------------------------------------------------
// GGUF block readers (blocks are 2-byte aligned: 18 B / 34 B).
// --------------------------------------------------------------------------
PI_DEV float gguf_scale(const uint8_t* blk) {
    return half_bits_to_float(*reinterpret_cast<const uint16_t*>(blk));
}
// int8 value i of a Q8_0 block
PI_DEV float q8_val(const uint8_t* blk, int i) { return (float)(int8_t)blk[2 + i]; }
// dequantised Q4_0 element i of a block (reference nibble order)
PI_DEV float q4_val(const uint8_t* blk, int i) {
    const uint8_t byte = blk[2 + (i >> 1)];
    const int nib = (i & 1) ? (byte >> 4) : (byte & 15);
    return (float)(nib - 8);
}

// element i of an F32 / Q4_0 / Q8_0 row, dequantised exactly as the reference
// (value * scale, f32 multiply).
PI_DEV float row_elem(const uint8_t* row, int qtype, int64_t i) {
    if (qtype == PI_QT_F32) return reinterpret_cast<const float*>(row)[i];
    if (qtype == PI_QT_Q4_0) {
        const uint8_t* blk = row + (i >> 5) * 18;
        return fmul(q4_val(blk, (int)(i & 31)), gguf_scale(blk));
    }
    const uint8_t* blk = row + (i >> 5) * 34;
    return fmul(q8_val(blk, (int)(i & 31)), gguf_scale(blk));
}

PI_DEV int64_t row_bytes(int qtype, int64_t n) {
    return qtype == PI_QT_F32 ? n * 4 : (qtype == PI_QT_Q4_0 ? n / 32 * 18 : n / 32 * 34);
}

// --------------------------------------------------------------------------
// Q8_0 activation quantiser over a vector (warp per 32-block).
// --------------------------------------------------------------------------
__global__ void k_quant_act(const float* __restrict__ x, int64_t n, int8_t* __restrict__ xq, float* __restrict__ xs) {
    const int64_t b = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b * 32 >= n) return;
    const int64_t i = b * 32 + lane;
    float sc;
    const int8_t q = warp_quant_q8(i < n ? x[i] : 0.0f, &sc);
    xq[i] = q;
    if (lane == 0) xs[b] = sc;
}

// --------------------------------------------------------------------------
// Q8_0 int-dot rows (matvec_col_major_q8_0, quant/mod.rs:652-689): warp per
// output row; lanes compute per-block integer dots; lane 0 then adds the
// block terms (float)sumi * (d_w * d_x) sequentially, blocks ascending.
// rows: idx == null -> row j; else row idx[j] (range-checked).
// --------------------------------------------------------------------------
__global__ __launch_bounds__(256) void k_rows_q8(float* __restrict__ y, const int8_t* __restrict__ xq,
                                                 const float* __restrict__ xs, const uint8_t* __restrict__ raw,
                                                 int64_t n_in, int64_t n_out, const int64_t* __restrict__ idx,
                                                 int64_t n_rows, uint32_t* err) {
    extern __shared__ float terms[];  // [8 warps][nb]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t j = blockIdx.x * 8LL + warp;
    if (j >= n_rows) return;
    int64_t r = j;
    if (idx) {
        r = idx[j];
        if (r < 0 || r >= n_out) {
            if (lane == 0) atomicOr(err, PI_DEVERR_INDEX);
            return;
        }
    }
    const int64_t nb = n_in / 32;
    float* tw = terms + warp * nb;
    const uint8_t* row = raw + r * nb * 34;
    for (int64_t b = lane; b < nb; b += 32) {
        const uint8_t* blk = row + b * 34;
        const uint16_t* q16 = reinterpret_cast<const uint16_t*>(blk + 2);
        const int* xi = reinterpret_cast<const int*>(xq + b * 32);
        int s = 0;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const uint32_t lo = q16[2 * m], hi = q16[2 * m + 1];
            s = dp4a((int)(lo | (hi << 16)), xi[m], s);
        }
        tw[b] = fmul((float)s, fmul(gguf_scale(blk), xs[b]));
    }
    __syncwarp();
    if (lane == 0) {
        float sum = 0.0f;
        for (int64_t b = 0; b < nb; ++b) sum = fadd(sum, tw[b]);
        y[j] = sum;
    }
}

// --------------------------------------------------------------------------
// f32-activation rows (F32 weights, or any type through the reference's
// dequantise-then-dot fallback, quant/mod.rs:958-969): thread per output row,
// sum = sum + x[i] * w[i], i ascending.
// --------------------------------------------------------------------------
__global__ __launch_bounds__(128) void k_rows_f32(float* __restrict__ y, const float* __restrict__ x,
                                                  const uint8_t* __restrict__ raw, int qtype, int64_t n_in,
                                                  int64_t n_out, const int64_t* __restrict__ idx, int64_t n_rows,
                                                  uint32_t* err) {
    __shared__ float xs[1024];
    const int64_t j = blockIdx.x * 128LL + threadIdx.x;
    int64_t r = j;
    bool ok = j < n_rows;
    if (ok && idx) {
        r = idx[j];
        if (r < 0 || r >= n_out) {
            atomicOr(err, PI_DEVERR_INDEX);
            ok = false;
        }
    }
    const uint8_t* row = raw + (ok ? r : 0) * row_bytes(qtype, n_in);
    float sum = 0.0f;
    for (int64_t c0 = 0; c0 < n_in; c0 += 1024) {
        __syncthreads();
        for (int i = threadIdx.x; i < 1024; i += 128) xs[i] = (c0 + i < n_in) ? x[c0 + i] : 0.0f;
        __syncthreads();
        if (!ok) continue;
        const int64_t lim = min((int64_t)1024, n_in - c0);
        for (int64_t i = 0; i < lim; ++i) sum = fadd(sum, fmul(xs[i], row_elem(row, qtype, c0 + i)));
    }
    if (ok) y[j] = sum;
}

// --------------------------------------------------------------------------
// sparse-input matvec (quant/mod.rs:1073-1169): thread per output c,
// sum = sum + x[s] * w[c][idx[s]] over s ascending (x NOT quantised).
// --------------------------------------------------------------------------
__global__ __launch_bounds__(128) void k_sparse_input(float* __restrict__ y, const float* __restrict__ x,
                                                      const int64_t* __restrict__ idx, int64_t n_idx,
                                                      const uint8_t* __restrict__ raw, int qtype, int64_t n_in,
                                                      int64_t n_out, uint32_t* err) {
    __shared__ float xs[512];
    __shared__ int64_t is[512];
    const int64_t c = blockIdx.x * 128LL + threadIdx.x;
    const uint8_t* row = raw + (c < n_out ? c : 0) * row_bytes(qtype, n_in);
    float sum = 0.0f;
    bool bad = false;
    for (int64_t s0 = 0; s0 < n_idx; s0 += 512) {
        __syncthreads();
        for (int i = threadIdx.x; i < 512; i += 128) {
            xs[i] = (s0 + i < n_idx) ? x[s0 + i] : 0.0f;
            is[i] = (s0 + i < n_idx) ? idx[s0 + i] : 0;
        }
        __syncthreads();
        const int64_t lim = min((int64_t)512, n_idx - s0);
        for (int64_t s = 0; s < lim; ++s) {
            const int64_t r = is[s];
            if (r < 0 || r >= n_in) { bad = true; continue; }
            sum = fadd(sum, fmul(xs[s], row_elem(row, qtype, r)));
        }
    }
    if (bad && threadIdx.x == 0) atomicOr(err, PI_DEVERR_INDEX);
    if (c < n_out) y[c] = sum;
}

__global__ void k_swiglu_vec(float* __restrict__ g, const float* __restrict__ u, int64_t n) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) g[i] = swiglu_ref(g[i], u[i]);
}

__global__ void k_dequant(const uint8_t* __restrict__ raw, int qtype, int64_t n, float* __restrict__ out) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (qtype == PI_QT_F16) out[i] = half_bits_to_float(reinterpret_cast<const uint16_t*>(raw)[i]);
    else out[i] = row_elem(raw, qtype, i);
}

// --------------------------------------------------------------------------
// Weight quantisers -> GGUF blocks. Warp per block.
// --------------------------------------------------------------------------
__global__ void k_quant_q8_blocks(const float* __restrict__ x, int64_t nblk, uint8_t* __restrict__ out) {
    const int64_t b = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= nblk) return;
    float sc;
    const int8_t q = warp_quant_q8(x[b * 32 + lane], &sc);
    // the 34-byte block as 17 little-endian u16 words: word 0 = f16 scale,
    // word j >= 1 = (q[2j-2], q[2j-1]); block starts are 2-byte aligned.
    const uint32_t qb = (uint8_t)q;
    const uint32_t lo = __shfl_sync(0xffffffffu, qb, (2 * lane - 2) & 31);
    const uint32_t hi = __shfl_sync(0xffffffffu, qb, (2 * lane - 1) & 31);
    uint16_t* o = reinterpret_cast<uint16_t*>(out + b * 34);
    if (lane == 0) o[0] = __half_as_ushort(__float2half_rn(sc));
    else if (lane < 17) o[lane] = (uint16_t)(lo | (hi << 8));
}

// ggml-style Q4_0: m = first element with the largest |x|; d = m / -8;
// id = 1/d; q = min(15, (int8)(x*id + 8.5)); packed byte i = q[2i] | q[2i+1] << 4.
__global__ void k_quant_q4_blocks(const float* __restrict__ x, int64_t nblk, uint8_t* __restrict__ out) {
    const int64_t b = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= nblk) return;
    const float v = x[b * 32 + lane];
    float ba = fabsf(v);
    if (ba != ba) ba = -1.0f;
    int bi = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, ba, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oa > ba || (oa == ba && oi < bi)) { ba = oa; bi = oi; }
    }
    const float m = __shfl_sync(0xffffffffu, v, bi);
    const float dd = fdiv(m, -8.0f);
    const float id = (dd != 0.0f) ? fdiv(1.0f, dd) : 0.0f;
    const float t = truncf(fadd(fmul(v, id), 8.5f));
    int q = (int)fminf(15.0f, fmaxf(0.0f, t));
    // packed byte i = q[2i] | q[2i+1] << 4; the 18-byte block as 9 u16 words:
    // word 0 = f16 scale, word j >= 1 = (byte 2j-2, byte 2j-1) = q[4j-4 .. 4j-1]
    const int q0 = __shfl_sync(0xffffffffu, q, (4 * lane - 4) & 31);
    const int q1 = __shfl_sync(0xffffffffu, q, (4 * lane - 3) & 31);
    const int q2 = __shfl_sync(0xffffffffu, q, (4 * lane - 2) & 31);
    const int q3 = __shfl_sync(0xffffffffu, q, (4 * lane - 1) & 31);
    uint16_t* o = reinterpret_cast<uint16_t*>(out + b * 18);
    if (lane == 0) o[0] = __half_as_ushort(__float2half_rn(dd));
    else if (lane < 9) o[lane] = (uint16_t)((q0 | (q1 << 4)) | ((q2 | (q3 << 4)) << 8));
}

// --------------------------------------------------------------------------
// Synthetic normals: SplitMix64 (model/mod.rs:2041-2061) + Box-Muller.
// --------------------------------------------------------------------------
__host__ __device__ inline uint64_t splitmix_at(uint64_t seed, uint64_t j) {
    uint64_t z = seed + (j + 1) * 0x9E3779B97F4A7C15ull;  // state after j+1 steps
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void k_synth(uint64_t seed, uint64_t offset, int64_t n, float stdv, float* __restrict__ out) {
    const int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (k >= n) return;
    const uint64_t i = offset + (uint64_t)k;
    const uint64_t m = i >> 1;
    const double u1 = 1.0 - (double)(splitmix_at(seed, 2 * m) >> 11) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(splitmix_at(seed, 2 * m + 1) >> 11) * (1.0 / 9007199254740992.0);
    const double r = sqrt(-2.0 * log(u1));
    const double th = 6.283185307179586 * u2;
    const double v = (i & 1) ? r * sin(th) : r * cos(th);
    out[k] = (float)(v * (double)stdv);
}

// --------------------------------------------------------------------------
// Predictor MLP (predictor/mod.rs:63-84): thread per output unit.
// --------------------------------------------------------------------------
__global__ void k_pred_layer(const float* __restrict__ in, int64_t T, int64_t n_in, const float* __restrict__ W,
                             const float* __restrict__ b, int64_t n_out, int act, float* __restrict__ out) {
    const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t t = blockIdx.y;
    if (j >= n_out || t >= T) return;
    const float* a = in + t * n_in;
    const float* w = W + j * n_in;
    float s = 0.0f;
    for (int64_t i = 0; i < n_in; ++i) s = fadd(s, fmul(w[i], a[i]));
    s = fadd(s, b[j]);
    out[t * n_out + j] = act == 0 ? fmaxf(s, 0.0f) : sigmoid_ref(s);
}

// --------------------------------------------------------------------------
// Hot-neuron sparse FFN (C-ABI pi_sparse_ffn_*).
// --------------------------------------------------------------------------
constexpr int SF_TMAX = 8;             // tokens per pass (one byte of mask bits per neuron)
constexpr int64_t SF_MAX_FF = 131072;  // neurons a layer may have
constexpr int SF_GU_WARPS = 16;        // warps of a gate/up CTA (one CTA per SM)

// Tokens t of the pass whose list covers all n_ff neurons take every neuron
// (quant/mod.rs:1221-1223): their bits, one per token.
PI_DEV uint32_t sf_dense_bits(const int64_t* __restrict__ ptr, int t0, int nt, int64_t n_ff) {
    uint32_t dense = 0;
    for (int t = 0; t < nt; ++t)
        if (ptr[t0 + t + 1] - ptr[t0 + t] >= n_ff) dense |= 1u << t;
    return dense;
}

// Marks the pass's (token, neuron) pairs: bit t of mask byte s = neuron s in token
// t0 + t's list, and zeroes h of the pass. The mask starts zero; the down kernel
// clears it (with coalesced stores, after gate/up has read it) and resets the
// counters, so both are zero again for the next pass. The first mark of a neuron
// appends it to the work list (wctr[0] = its length), which the gate/up warps drain.
__global__ __launch_bounds__(256) void k_sf_mark(const int64_t* __restrict__ ptr, const int64_t* __restrict__ idx,
                                                 int t0, int nt, int64_t n_ff, uint32_t* __restrict__ mask32,
                                                 int32_t* __restrict__ wlist, uint32_t* __restrict__ wctr,
                                                 float* __restrict__ h, uint32_t* __restrict__ err) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    int64_t bnd[SF_TMAX + 1];
#pragma unroll
    for (int t = 0; t <= SF_TMAX; ++t) bnd[t] = t <= nt ? ptr[t0 + t] : 0;
    const int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, gsz = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = gid; i < nt * n_ff / 4; i += gsz) reinterpret_cast<float4*>(h)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t e = bnd[0] + gid; e < bnd[nt]; e += gsz) {
        int t = 0;
        while (e >= bnd[t + 1]) ++t;
        const int64_t sn = idx[e];
        if (sn < 0 || sn >= n_ff) {
            atomicOr(err, PI_DEVERR_INDEX);
            continue;
        }
        const uint32_t old = atomicOr(&mask32[sn >> 2], 1u << (8 * (sn & 3) + t));
        if (((old >> (8 * (sn & 3))) & 0xFFu) == 0) wlist[atomicAdd(&wctr[0], 1u)] = (int32_t)sn;
    }
}

PI_DEV float nibf(uint32_t v) { return __int_as_float(0x4B000000u | v) - 8388616.0f; }
// packed f32x2 helpers (sm_100 FADD2 / FFMA2 on register pairs)
PI_DEV uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
PI_DEV uint64_t f2_pack_u(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
PI_DEV void f2_unpack(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
PI_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
PI_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// gate/up of every marked (token, neuron) pair, h = SwiGLU(g, u) (quant/mod.rs:1196-1199)
// into h[t][n] (0 where the pair is not marked); the pass's output rows are zeroed
// for the down kernel's atomics. Persistent: one CTA per SM stages the pass's
// activations once; warp w walks neurons w, w + W, ... and streams each marked
// neuron's gate and up rows once for all of its tokens.
// Q4_0: x f32, staged with 32-float blocks 36 floats apart (lane l reads blocks
// l + 32 j with float4 loads in distinct banks); the reference dequantises the
// whole matrix and sums in f32 (quant/mod.rs:958-969).
// Q8_0: x quantised to Q8_0 (quant/mod.rs:698-736), int8 block dots, block terms
// (float)sumi * (d_w * d_x) (quant/mod.rs:819-899).
// DIRECT (one token, the fused pass): the work items are the token's own list
// entries, read straight from idx; a neuron listed twice is computed once (the
// first claim sets its mask bit, a later claim that finds the bit set skips it),
// and out-of-range entries set PI_DEVERR_INDEX and are skipped.
template <int QT, int BPL, int NTM, bool DIRECT>
PI_DEV void sf_gateup_body(const uint8_t* __restrict__ G, const uint8_t* __restrict__ U, const __half* __restrict__ GD,
                           const __half* __restrict__ UD, uint8_t* __restrict__ mask, const float* __restrict__ x,
                           const int8_t* __restrict__ xq, const float* __restrict__ xs,
                           const int64_t* __restrict__ ptr, const int64_t* __restrict__ idx,
                           const int32_t* __restrict__ wlist, uint32_t* __restrict__ wctr, int t0, int nt,
                           int64_t n_ff, float* __restrict__ h, float* __restrict__ y, uint32_t* __restrict__ err,
                           float* __restrict__ sf_x) {
    static_assert(!DIRECT || NTM == 1, "list entries as work items: one token per pass");
    constexpr int NB = 32 * BPL;  // blocks per row
    constexpr int64_t D = 32 * NB;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // stage the pass's activations; zero its output rows (run after the first rows are requested)
    auto stage_x = [&]() {
    if (QT == PI_QT_Q4_0) {
        for (int k = tid; k < nt * (int)D / 4; k += blockDim.x) {
            const int t = k / ((int)D / 4), r = k % ((int)D / 4);
            const float4 v = reinterpret_cast<const float4*>(x + (int64_t)(t0 + t) * D)[r];
            *reinterpret_cast<float4*>(&sf_x[(size_t)t * NB * 36 + 36 * (r >> 3) + 4 * (r & 7)]) = v;
        }
    } else {
        int8_t* s8 = reinterpret_cast<int8_t*>(sf_x);
        float* ssc = sf_x + nt * D / 4;
        for (int k = tid; k < nt * (int)D / 16; k += blockDim.x)
            reinterpret_cast<int4*>(s8)[k] = reinterpret_cast<const int4*>(xq + (int64_t)t0 * D)[k];
        for (int k = tid; k < nt * NB; k += blockDim.x) ssc[k] = xs[(int64_t)t0 * NB + k];
    }
    {
        float4* o4 = reinterpret_cast<float4*>(y + (int64_t)t0 * D);
        for (int64_t k = blockIdx.x * (int64_t)blockDim.x + tid; k < nt * D / 4; k += (int64_t)gridDim.x * blockDim.x)
            o4[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    };
    const uint32_t dense = sf_dense_bits(ptr, t0, nt, n_ff);
    constexpr int WPB = QT == PI_QT_Q4_0 ? 1 : 2;  // 16-byte words per block
    // Work: the neurons the pass marked (the work list), or every neuron when a token's
    // list is complete. Warps claim one neuron at a time from a counter (a claimed
    // neuron runs for all of its tokens), so the load follows the work as it comes.
    // The first item of warp w is item w (no atomic); later ones are W + the counter.
    // (the list length is read through L2: in the fused pass other CTAs wrote it)
    const int64_t p0 = DIRECT ? ptr[t0] : 0;
    const uint32_t n_items = dense ? (uint32_t)n_ff
                                   : (DIRECT ? (uint32_t)(ptr[t0 + 1] - p0) : __ldcg(&wctr[0]));
    const uint32_t W = gridDim.x * SF_GU_WARPS;
    bool first = true;
    auto claim = [&]() -> int64_t {
        for (;;) {
            uint32_t i = n_items;
            if (first) {
                i = blockIdx.x * SF_GU_WARPS + warp;
                first = false;
            } else if (n_items > W && lane == 0 && W + *reinterpret_cast<volatile uint32_t*>(&wctr[1]) < n_items) {
                i = W + atomicAdd(&wctr[1], 1u);
            }
            i = __shfl_sync(0xffffffffu, i, 0);
            if (i >= n_items) return -1;
            if (dense) return (int64_t)i;
            if (!DIRECT) return (int64_t)__ldcg(&wlist[i]);
            const int64_t sn = idx[p0 + i];
            if (sn >= 0 && sn < n_ff) return sn;
            if (lane == 0) atomicOr(err, PI_DEVERR_INDEX);
        }
    };
    // DIRECT: the claim that sets neuron n's mask bit computes it; a repeated entry skips
    auto repeated = [&](int64_t n) -> bool {
        if (!DIRECT || dense) return false;
        uint32_t old = 0;
        if (lane == 0) old = atomicOr(reinterpret_cast<uint32_t*>(mask) + (n >> 2), 1u << (8 * (n & 3)));
        return (__shfl_sync(0xffffffffu, old, 0) >> (8 * (n & 3))) & 1u;
    };
    int4 wg[BPL][WPB], wu[BPL][WPB];
    float dg[BPL], du[BPL];
    auto load = [&](int64_t n) {
#pragma unroll
        for (int j = 0; j < BPL; ++j) {
            const int b = lane + 32 * j;
#pragma unroll
            for (int k = 0; k < WPB; ++k) {
                wg[j][k] = ld_stream(G + n * (D * WPB / 2) + (int64_t)b * 16 * WPB + 16 * k);
                wu[j][k] = ld_stream(U + n * (D * WPB / 2) + (int64_t)b * 16 * WPB + 16 * k);
            }
            dg[j] = __half2float(GD[n * NB + b]);
            du[j] = __half2float(UD[n * NB + b]);
        }
    };
    int64_t nxt = claim();
    bool nxt_rep = false;
    if (nxt >= 0) {
        load(nxt);
        nxt_rep = repeated(nxt);
    }
    stage_x();  // while the first rows are in flight
    __syncthreads();
    while (nxt >= 0) {
        const int64_t n = nxt;
        const bool rep = nxt_rep;
        uint32_t m = 1;  // one token: every listed neuron is its own (no mask read to wait for)
        if (NTM != 1) {
            if (lane == 0) m = (__ldcg(&mask[n]) | dense) & ((1u << nt) - 1u);
            m = __shfl_sync(0xffffffffu, m, 0);
        }
        if (rep) m = 0;
        nxt = claim();
        {
            // this neuron's rows are in registers: compute every marked token
            float part_g[NTM], part_u[NTM];
#pragma unroll
            for (int t = 0; t < NTM; ++t) part_g[t] = part_u[t] = 0.f;
            if (QT == PI_QT_Q4_0) {
                // each nibble is decoded once and used by every marked token
#pragma unroll
                for (int j = 0; j < BPL; ++j) {
                    const int b = lane + 32 * j;
                    // packed pair accumulators: (element 2k, element 2k + 1) of each token
                    uint64_t bg2[NTM], bu2[NTM];
#pragma unroll
                    for (int t = 0; t < NTM; ++t) bg2[t] = bu2[t] = 0ull;
                    uint32_t g0 = wg[j][0].x, g1 = wg[j][0].y, g2 = wg[j][0].z, g3 = wg[j][0].w;
                    uint32_t u0 = wu[j][0].x, u1 = wu[j][0].y, u2 = wu[j][0].z, u3 = wu[j][0].w;
                    const uint64_t off8 = f2_pack(-8388616.0f, -8388616.0f);
#pragma unroll 1
                    for (int i = 0; i < 4; ++i) {  // word i = elements 8i .. 8i+7 (byte k: 2k low, 2k+1 high)
                        // nibbles -> f32 (n - 8): byte k of the low / high nibble planes under the
                        // exponent of 2^23, minus 2^23 + 8, two at a time
                        uint64_t fg[4], fu[4];
                        const uint32_t gl = g0 & 0x0F0F0F0Fu, gh = (g0 >> 4) & 0x0F0F0F0Fu;
                        const uint32_t ul = u0 & 0x0F0F0F0Fu, uh = (u0 >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            fg[k] = f2_add(f2_pack_u(__byte_perm(gl, 0x4B000000u, 0x7440 + k),
                                                     __byte_perm(gh, 0x4B000000u, 0x7440 + k)), off8);
                            fu[k] = f2_add(f2_pack_u(__byte_perm(ul, 0x4B000000u, 0x7440 + k),
                                                     __byte_perm(uh, 0x4B000000u, 0x7440 + k)), off8);
                        }
#pragma unroll
                        for (int t = 0; t < NTM; ++t) {
                            if (t >= nt || !((m >> t) & 1u)) continue;
                            const float* xb = sf_x + (size_t)t * NB * 36 + 36 * b + 8 * i;
                            const float4 xa = *reinterpret_cast<const float4*>(xb);
                            const float4 xc = *reinterpret_cast<const float4*>(xb + 4);
                            const uint64_t xp[4] = {f2_pack(xa.x, xa.y), f2_pack(xa.z, xa.w), f2_pack(xc.x, xc.y),
                                                    f2_pack(xc.z, xc.w)};
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                bg2[t] = f2_fma(fg[k], xp[k], bg2[t]);
                                bu2[t] = f2_fma(fu[k], xp[k], bu2[t]);
                            }
                        }
                        g0 = g1; g1 = g2; g2 = g3;
                        u0 = u1; u1 = u2; u2 = u3;
                    }
                    float bg[NTM], bu[NTM];
#pragma unroll
                    for (int t = 0; t < NTM; ++t) {
                        float a0, a1, c0, c1;
                        f2_unpack(bg2[t], a0, a1);
                        f2_unpack(bu2[t], c0, c1);
                        bg[t] = a0 + a1;
                        bu[t] = c0 + c1;
                    }
#pragma unroll
                    for (int t = 0; t < NTM; ++t) {
                        part_g[t] += dg[j] * bg[t];
                        part_u[t] += du[j] * bu[t];
                    }
                }
            } else {
#pragma unroll
                for (int t = 0; t < NTM; ++t) {
                    if (t >= nt || !((m >> t) & 1u)) continue;
                    float sg = 0.f, su = 0.f;
#pragma unroll
                    for (int j = 0; j < BPL; ++j) {
                        const int b = lane + 32 * j;
                        const int8_t* s8 = reinterpret_cast<const int8_t*>(sf_x) + (size_t)t * D + 32 * b;
                        const float dxv = sf_x[nt * D / 4 + t * NB + b];
                        const int4 xa = *reinterpret_cast<const int4*>(s8), xc = *reinterpret_cast<const int4*>(s8 + 16);
                        int ag = dp4a(wg[j][0].x, xa.x, 0), au = dp4a(wu[j][0].x, xa.x, 0);
                        ag = dp4a(wg[j][0].y, xa.y, ag); au = dp4a(wu[j][0].y, xa.y, au);
                        ag = dp4a(wg[j][0].z, xa.z, ag); au = dp4a(wu[j][0].z, xa.z, au);
                        ag = dp4a(wg[j][0].w, xa.w, ag); au = dp4a(wu[j][0].w, xa.w, au);
                        ag = dp4a(wg[j][WPB - 1].x, xc.x, ag); au = dp4a(wu[j][WPB - 1].x, xc.x, au);
                        ag = dp4a(wg[j][WPB - 1].y, xc.y, ag); au = dp4a(wu[j][WPB - 1].y, xc.y, au);
                        ag = dp4a(wg[j][WPB - 1].z, xc.z, ag); au = dp4a(wu[j][WPB - 1].z, xc.z, au);
                        ag = dp4a(wg[j][WPB - 1].w, xc.w, ag); au = dp4a(wu[j][WPB - 1].w, xc.w, au);
                        sg += (float)ag * (dg[j] * dxv);
                        su += (float)au * (du[j] * dxv);
                    }
                    part_g[t] = sg;
                    part_u[t] = su;
                }
            }
            // the next marked neuron's rows are requested before the reductions
            if (nxt >= 0) {
                load(nxt);
                nxt_rep = repeated(nxt);
            }
            float hv = 0.f;  // lane t keeps token t's h
#pragma unroll
            for (int t = 0; t < NTM; ++t) {
                if (t >= nt || !((m >> t) & 1u)) continue;
                const float sg = warp_sum(part_g[t]), su = warp_sum(part_u[t]);
                if (lane == t) hv = swiglu_ref(sg, su);
            }
            if (lane < nt && !rep) h[(int64_t)lane * n_ff + n] = hv;
        }
    }
}

template <int QT, int BPL, int NTM>  // BPL: blocks per lane (n_embd = 32 * 32 * BPL); NTM: tokens (1 or 8)
__global__ __launch_bounds__(SF_GU_WARPS * 32, 1) void k_sf_gateup(
    const uint8_t* __restrict__ G, const uint8_t* __restrict__ U, const __half* __restrict__ GD,
    const __half* __restrict__ UD, uint8_t* __restrict__ mask, const float* __restrict__ x,
    const int8_t* __restrict__ xq, const float* __restrict__ xs, const int64_t* __restrict__ ptr,
    const int32_t* __restrict__ wlist, uint32_t* __restrict__ wctr, int t0, int nt, int64_t n_ff,
    float* __restrict__ h, float* __restrict__ y) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    extern __shared__ __align__(16) float sf_x[];
    sf_gateup_body<QT, BPL, NTM, false>(G, U, GD, UD, mask, x, xq, xs, ptr, nullptr, wlist, wctr, t0, nt, n_ff, h, y,
                                        nullptr, sf_x);
}

// down, neuron-major, of the pass: CTA = (512 output columns, 64 neurons), thread =
// 2 consecutive columns. The CTA loads h of its neurons for every token, keeps the
// neurons with any nonzero h, copies their weight slices into shared memory
// (cp.async) while it loads the block scales, then runs over them; y gets float2
// atomics. Q8_0 weights and a token whose list is complete: the reference then takes
// the dense ffn_swiglu_q, whose down projection re-quantises h to Q8_0 blocks
// (quant/mod.rs:1203), so such a token's h is replaced by its Q8_0 value q * d.
constexpr int SF_DN = 64;  // neurons per down CTA (two 32-neuron scale groups)
template <int QT, int NTM>
__global__ __launch_bounds__(256) void k_sf_down(const uint8_t* __restrict__ DQ, const __half* __restrict__ DS,
                                                 const float* __restrict__ h, const int64_t* __restrict__ ptr, int t0,
                                                 int nt, int64_t n_embd, int64_t n_ff, float* __restrict__ y,
                                                 uint32_t* __restrict__ wctr, uint8_t* __restrict__ mask) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    __shared__ float s_h[NTM][SF_DN];
    __shared__ int32_t s_list[SF_DN];
    __shared__ int s_cnt[2];
    __shared__ float2 s_sc[SF_DN / 32][256];
    constexpr int RB = QT == PI_QT_Q4_0 ? 256 : 512;  // bytes of a neuron's 512 columns
    __shared__ __align__(16) uint8_t s_w[SF_DN][RB];
    const int64_t n0 = (int64_t)blockIdx.y * SF_DN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t c = blockIdx.x * 512LL + 2 * tid;
    if (blockIdx.x == 0 && blockIdx.y == 0 && tid == 0) wctr[0] = wctr[1] = 0;  // gate/up has drained the list
    // the pass's marks are read: clear this neuron group's mask bytes for the next pass
    if (blockIdx.x == 0 && tid < SF_DN / 16 && n0 + 16 * (tid + 1) <= n_ff)
        reinterpret_cast<uint4*>(mask + n0)[tid] = make_uint4(0, 0, 0, 0);
    if (tid < SF_DN) {
#pragma unroll
        for (int t = 0; t < NTM; ++t) s_h[t][tid] = (t < nt && n0 + tid < n_ff) ? h[(int64_t)t * n_ff + n0 + tid] : 0.f;
    }
    __syncthreads();
    if (QT == PI_QT_Q8_0 && warp < SF_DN / 32) {
        for (int t = 0; t < nt && t < NTM; ++t) {
            if (ptr[t0 + t + 1] - ptr[t0 + t] < n_ff) continue;
            float sc;
            const int8_t q = warp_quant_q8(s_h[t][32 * warp + lane], &sc);
            s_h[t][32 * warp + lane] = fmul((float)q, sc);
        }
    }
    if (warp < SF_DN / 32) {  // the neurons with any nonzero h, ascending
        bool any = false;
#pragma unroll
        for (int t = 0; t < NTM; ++t) any |= s_h[t][32 * warp + lane] != 0.f;
        const uint32_t bal = __ballot_sync(0xffffffffu, any);
        if (lane == 0) s_cnt[warp] = __popc(bal);
        __syncwarp();
        __shared__ uint32_t s_bal[SF_DN / 32];
        if (lane == 0) s_bal[warp] = bal;
        __syncwarp();
        asm volatile("bar.sync 1, 64;" ::: "memory");
        const int base = warp ? s_cnt[0] : 0;
        if (any) s_list[base + __popc(bal & ((1u << lane) - 1u))] = 32 * warp + lane;
    }
    __syncthreads();
    const int n = s_cnt[0] + s_cnt[1];
    if (n == 0) return;
    {
        const int64_t rowb = QT == PI_QT_Q4_0 ? n_embd / 2 : n_embd;
        const int64_t cb = blockIdx.x * (int64_t)RB;
        for (int q = tid; q < n * (RB / 16); q += 256) {
            const int i = q / (RB / 16), ch = q % (RB / 16);
            const uint32_t sa = (uint32_t)__cvta_generic_to_shared(&s_w[i][16 * ch]);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa),
                         "l"(DQ + (n0 + s_list[i]) * rowb + cb + 16 * ch)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
#pragma unroll
    for (int gi = 0; gi < SF_DN / 32; ++gi) {
        float2 sc = make_float2(0.f, 0.f);
        if (s_cnt[gi] > 0)
            sc = __half22float2(*reinterpret_cast<const __half2*>(DS + ((n0 >> 5) + gi) * n_embd + c));
        s_sc[gi][tid] = sc;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    float acc[NTM][2];
#pragma unroll
    for (int t = 0; t < NTM; ++t) acc[t][0] = acc[t][1] = 0.f;
#pragma unroll 8
    for (int i = 0; i < n; ++i) {
        const int sl = s_list[i];
        const float2 sc = s_sc[sl >> 5][tid];
        float w0, w1;
        if (QT == PI_QT_Q4_0) {
            const uint32_t v = s_w[i][tid];
            w0 = nibf(v & 15u) * sc.x;
            w1 = nibf(v >> 4) * sc.y;
        } else {
            const uint32_t v = *reinterpret_cast<const uint16_t*>(&s_w[i][2 * tid]);
            w0 = (float)(int8_t)(v & 0xffu) * sc.x;
            w1 = (float)(int8_t)(v >> 8) * sc.y;
        }
#pragma unroll
        for (int t = 0; t < NTM; ++t) {
            const float hv = s_h[t][sl];
            acc[t][0] += hv * w0;
            acc[t][1] += hv * w1;
        }
    }
#pragma unroll
    for (int t = 0; t < NTM; ++t)
        if (t < nt && (acc[t][0] != 0.f || acc[t][1] != 0.f))
            atomicAdd(reinterpret_cast<float2*>(y + (int64_t)(t0 + t) * n_embd + c), make_float2(acc[t][0], acc[t][1]));
}

// ---------------------------------------------------------------------------
// A one-token sparse-FFN pass in one persistent kernel (one CTA of 512 threads per
// SM, every CTA resident): gate/up -> grid barrier -> down. It computes what
// k_sf_mark, k_sf_gateup and k_sf_down compute for one token, without their launch
// gaps: gate/up warps take the token's list entries straight from idx (a repeated
// entry is computed once: the first claim sets the neuron's mask bit), and each
// CTA prefetches the down block scales of its first unit while gate/up runs.
// (Passes of several tokens keep the three launches: measured, a mark phase and a
// second barrier inside one kernel cost more than the launches they replace.)
//
// Down work unit = (512 output columns, a range of RN consecutive neurons, RN a
// multiple of 32 so the range holds whole 32-neuron scale groups). The unit finds
// its active neurons from the mask (every neuron when the token's list is
// complete), stages their weight slices by cp.async in
// double-buffered chunks (as many neurons as the shared memory left by gate/up
// holds, at least 128), sums them in two halves of 256 threads (2 columns a
// thread, packed f32x2 fused multiply-adds) and adds the result to y with float2
// atomics. The last of the
// n_embd / 512 units of a range to read the range's mask clears it (a ticket per
// range), so the mask is zero again for the next pass; CTA 0 resets the work-list
// counters after the second barrier.
// ---------------------------------------------------------------------------
struct SfGridBar {
    uint32_t count, gen;
};

// Grid-wide barrier for a kernel whose CTAs are all resident: the last CTA to
// arrive resets the count and advances the generation the others wait on. The
// wait is bounded (2^24 polls, the later ones 32 ns apart: about half a second);
// when it runs out, the kernel
// records PI_DEVERR_TIMEOUT and every CTA returns.
PI_DEV bool sf_grid_sync(SfGridBar* g, uint32_t* err, int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        volatile uint32_t* gen = &g->gen;
        const uint32_t g0 = *gen;
        __threadfence();
        if (atomicAdd(&g->count, 1u) == gridDim.x - 1) {
            atomicExch(&g->count, 0u);
            __threadfence();
            atomicAdd(&g->gen, 1u);
        } else {
            uint32_t it = 0;
            while (*gen == g0) {
                if (++it > (1u << 24)) {
                    ok = 0;
                    atomicOr(err, PI_DEVERR_TIMEOUT);
                    break;
                }
                if (it > 4096) __nanosleep(32);
            }
        }
        __threadfence();
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

struct SfFusedArgs {
    const uint8_t *G, *U;
    const __half *GD, *UD;
    const uint8_t* DQ;
    const __half* DS;
    uint8_t* mask;
    int32_t* wlist;
    uint32_t* wctr;
    uint32_t* tick;  // [n_ff / 32] per-range tickets, zero between passes
    SfGridBar* bar;
    const float* x;
    const int8_t* xq;
    const float* xs;
    const int64_t *ptr, *idx;
    int t0, nt, rn, fch;  // rn: neurons per down range; fch: neurons per down chunk (multiple of 32)
    int64_t n_embd, n_ff;
    float *h, *y;
    uint32_t* err;
    uint32_t stage_bytes;  // bytes of the staging region (x for gate/up, then the down chunks)
};

constexpr int SF_FT = 512;   // threads of a fused CTA
constexpr int SF_FMAXG = 32;  // scale groups per range (bounds the prefetched scales)

template <int QT, int BPL>
__global__ __launch_bounds__(SF_FT, 1) void k_sf_fused(const __grid_constant__ SfFusedArgs a) {
    constexpr int NTM = 1;
    static_assert(SF_GU_WARPS * 32 == SF_FT, "gate/up body runs on the fused CTA");
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    extern __shared__ __align__(16) uint8_t sf_sm[];
    constexpr int RB = QT == PI_QT_Q4_0 ? 256 : 512;  // bytes of one neuron's 512 columns
    __shared__ int s_ok, s_cnt[SF_FT / 32], s_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nt = a.nt;
    const int64_t n_ff = a.n_ff, d = a.n_embd;
    const int n_cc = (int)(d / 512), rn = a.rn;
    const int n_rng = (int)((n_ff + rn - 1) / rn), n_units = n_cc * n_rng;
    // dynamic shared memory: [staging | down chunk] [scales of a range] [active list]
    uint8_t* stage = sf_sm;
    __half2* s_sc = reinterpret_cast<__half2*>(sf_sm + a.stage_bytes);  // [group][256] column pairs
    uint32_t* s_act = reinterpret_cast<uint32_t*>(sf_sm + a.stage_bytes + SF_FMAXG * 1024);
    auto load_scales = [&](int u) {
        const int cc = u % n_cc;
        const int64_t s0 = (int64_t)(u / n_cc) * rn;
        const int ng = (int)(min((int64_t)rn, n_ff - s0) / 32);
        for (int q = tid; q < ng * 64; q += SF_FT) {  // 64 pieces of 16 bytes per group
            const int g = q >> 6, pc = q & 63;
            const uint32_t sa = (uint32_t)__cvta_generic_to_shared(reinterpret_cast<uint8_t*>(s_sc) + g * 1024 + 16 * pc);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa),
                         "l"(a.DS + (s0 / 32 + g) * d + cc * 512 + 8 * pc)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (blockIdx.x < n_units) load_scales(blockIdx.x);  // lands while gate/up runs

    const uint32_t tmask = 1u;
    // ---- gate/up (h of the listed neurons; the token's row of y zeroed)
    sf_gateup_body<QT, BPL, 1, true>(a.G, a.U, a.GD, a.UD, a.mask, a.x, a.xq, a.xs, a.ptr, a.idx, a.wlist, a.wctr,
                                     a.t0, nt, n_ff, a.h, a.y, a.err, reinterpret_cast<float*>(stage));
    if (!sf_grid_sync(a.bar, a.err, &s_ok)) return;
    pdl_trigger();  // every CTA is resident and past its last wait on the others
    if (blockIdx.x == 0 && tid == 0) a.wctr[0] = a.wctr[1] = 0;  // the list is drained
    const uint32_t dense = sf_dense_bits(a.ptr, a.t0, nt, n_ff);

    // ---- down
    const int fch = a.fch;                                                      // neurons per down chunk
    uint8_t* s_w = stage;                                                       // [2][fch][RB]
    float* s_h = reinterpret_cast<float*>(stage + 2 * fch * RB);               // [2][NTM][fch]
    float2* s_red = reinterpret_cast<float2*>(stage + 2 * fch * RB + 2 * NTM * fch * 4);  // [NTM][256]
    const int hf = tid >> 8, j = tid & 255;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const int cc = u % n_cc, r = u / n_cc;
        const int64_t s0 = (int64_t)r * rn;
        const int ns = (int)min((int64_t)rn, n_ff - s0);
        if (u != (int)blockIdx.x) {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            __syncthreads();  // the previous unit is done with the scales
            load_scales(u);
        }
        // active neurons of the range, ascending: entry = token bits << 16 | neuron offset
        int cnt = 0;
        uint32_t mine[2] = {0, 0};
        bool have[2] = {false, false};
        for (int k = 0; k < 2; ++k) {
            const int i = warp * 64 + 32 * k + lane;
            uint32_t bits = 0;
            if (i < ns) bits = ((uint32_t)__ldcg(&a.mask[s0 + i]) | dense) & tmask;
            have[k] = bits != 0;
            mine[k] = (bits << 16) | (uint32_t)i;
            cnt += __popc(__ballot_sync(0xffffffffu, have[k]));
        }
        if (lane == 0) s_cnt[warp] = cnt;
        __syncthreads();
        int base = 0, nact = 0;
        for (int w = 0; w < SF_FT / 32; ++w) {
            base += w < warp ? s_cnt[w] : 0;
            nact += s_cnt[w];
        }
        for (int k = 0; k < 2; ++k) {
            const uint32_t bal = __ballot_sync(0xffffffffu, have[k]);
            if (have[k]) s_act[base + __popc(bal & ((1u << lane) - 1u))] = mine[k];
            base += __popc(bal);
        }
        if (tid == 0) s_flag = atomicAdd(&a.tick[r], 1u) == (uint32_t)(n_cc - 1);
        __syncthreads();
        if (s_flag) {  // every unit of this range has read its mask: clear it for the next pass
            for (int i = tid; i < ns / 16; i += SF_FT)
                reinterpret_cast<uint4*>(a.mask + s0)[i] = make_uint4(0, 0, 0, 0);
            if (tid == 0) atomicExch(&a.tick[r], 0u);
        }
        const int64_t c = cc * 512LL + 2 * j;
        const int64_t rowb = QT == PI_QT_Q4_0 ? d / 2 : d;
        uint64_t acc[NTM];  // packed (column c, c + 1) sums per token
#pragma unroll
        for (int t = 0; t < NTM; ++t) acc[t] = 0ull;
        // chunks of fch active neurons, double-buffered: chunk k + 1's weight slices are
        // in flight while chunk k is summed
        auto issue = [&](int c0, int bf) {
            const int nc = min(fch, nact - c0);
            uint8_t* w = s_w + bf * (fch * RB);
            for (int q = tid; q < nc * (RB / 16); q += SF_FT) {
                const int i = q / (RB / 16), ch = q % (RB / 16);
                const int64_t sn = s0 + (s_act[c0 + i] & 0xffffu);
                const uint32_t sa = (uint32_t)__cvta_generic_to_shared(w + i * RB + 16 * ch);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa),
                             "l"(a.DQ + sn * rowb + cc * (int64_t)RB + 16 * ch)
                             : "memory");
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            for (int q = tid; q < NTM * fch; q += SF_FT) {
                const int t = q / fch, i = q % fch;
                float v = 0.f;
                if (t < nt && i < nc) {
                    const uint32_t e = s_act[c0 + i];
                    if ((e >> (16 + t)) & 1u) v = __ldcg(&a.h[(int64_t)t * n_ff + s0 + (e & 0xffffu)]);
                }
                s_h[(bf * NTM + t) * fch + i] = v;
            }
        };
        if (nact > 0) issue(0, 0);
        for (int c0 = 0, bf = 0; c0 < nact; c0 += fch, bf ^= 1) {
            const int nc = min(fch, nact - c0);
            if (c0 + fch < nact) {
                issue(c0 + fch, bf ^ 1);
                asm volatile("cp.async.wait_group 1;" ::: "memory");
            } else {
                asm volatile("cp.async.wait_group 0;" ::: "memory");
            }
            float* sh = s_h + bf * NTM * fch;
            const uint8_t* w = s_w + bf * (fch * RB);
            if (QT == PI_QT_Q8_0 && dense) {
                // a complete list takes the dense ffn_swiglu_q, which re-quantises h to Q8_0
                // (quant/mod.rs:1203); with a complete list every neuron is active, so the
                // chunk holds whole 32-neuron groups in order
                __syncthreads();
                for (int g = warp; 32 * g < nc; g += SF_FT / 32) {
                    for (int t = 0; t < nt && t < NTM; ++t) {
                        if (!((dense >> t) & 1u)) continue;
                        float sc;
                        const int8_t qv = warp_quant_q8(sh[t * fch + 32 * g + lane], &sc);
                        sh[t * fch + 32 * g + lane] = fmul((float)qv, sc);
                    }
                }
            }
            __syncthreads();
            for (int i = hf; i < nc; i += 2) {
                const int sl = (int)(s_act[c0 + i] & 0xffffu);
                const float2 sc = __half22float2(s_sc[(sl >> 5) * 256 + j]);
                float w0, w1;
                if (QT == PI_QT_Q4_0) {
                    const uint32_t v = w[i * RB + j];
                    w0 = nibf(v & 15u) * sc.x;
                    w1 = nibf(v >> 4) * sc.y;
                } else {
                    const uint32_t v = *reinterpret_cast<const uint16_t*>(&w[i * RB + 2 * j]);
                    w0 = (float)(int8_t)(v & 0xffu) * sc.x;
                    w1 = (float)(int8_t)(v >> 8) * sc.y;
                }
                const uint64_t w2 = f2_pack(w0, w1);
#pragma unroll
                for (int t = 0; t < NTM; ++t) {
                    const float hv = sh[t * fch + i];
                    acc[t] = f2_fma(w2, f2_pack(hv, hv), acc[t]);
                }
            }
            __syncthreads();  // the chunk's buffers are free
        }
        if (hf == 1) {
#pragma unroll
            for (int t = 0; t < NTM; ++t) {
                float v0, v1;
                f2_unpack(acc[t], v0, v1);
                s_red[t * 256 + j] = make_float2(v0, v1);
            }
        }
        __syncthreads();
        if (hf == 0) {
#pragma unroll
            for (int t = 0; t < NTM; ++t) {
                const float2 o = s_red[t * 256 + j];
                float v0, v1;
                f2_unpack(acc[t], v0, v1);
                v0 += o.x;
                v1 += o.y;
                if (t < nt && (v0 != 0.f || v1 != 0.f))
                    atomicAdd(reinterpret_cast<float2*>(a.y + (int64_t)(a.t0 + t) * d + c), make_float2(v0, v1));
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // a CTA without a unit may still own none
}

// Repack GGUF down [ne0=n_ff, ne1=n_embd] to neuron-major. Thread per
// (output pair c, c+1; block b of 32 neurons).
__global__ void k_repack_down_nm(const uint8_t* __restrict__ raw, int qtype, int64_t n_embd, int64_t n_ff,
                                 uint8_t* __restrict__ q, __half* __restrict__ sc) {
    const int64_t nb = n_ff / 32;
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t b = tid % nb, cp = tid / nb;
    const int64_t c = cp * 2;
    if (c >= n_embd) return;
    const int bsz = qtype == PI_QT_Q4_0 ? 18 : 34;
    const uint8_t* b0 = raw + (c * nb + b) * bsz;
    const uint8_t* b1 = raw + ((c + 1) * nb + b) * bsz;
    sc[b * n_embd + c] = __ushort_as_half(*reinterpret_cast<const uint16_t*>(b0));
    sc[b * n_embd + c + 1] = __ushort_as_half(*reinterpret_cast<const uint16_t*>(b1));
    for (int i = 0; i < 32; ++i) {
        const int64_t s = b * 32 + i;
        if (qtype == PI_QT_Q4_0) {
            const uint8_t v0 = b0[2 + (i >> 1)], v1 = b1[2 + (i >> 1)];
            const uint8_t n0 = (i & 1) ? (v0 >> 4) : (v0 & 15), n1 = (i & 1) ? (v1 >> 4) : (v1 & 15);
            q[s * (n_embd / 2) + c / 2] = (uint8_t)(n0 | (n1 << 4));
        } else {
            q[s * n_embd + c] = b0[2 + i];
            q[s * n_embd + c + 1] = b1[2 + i];
        }
    }
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
static int64_t gguf_size(int qtype, int64_t n) {
    switch (qtype) {
        case PI_QT_F32: return n * 4;
        case PI_QT_F16: return n * 2;
        case PI_QT_Q4_0: return n / 32 * 18;
        case PI_QT_Q8_0: return n / 32 * 34;
    }
    return -1;
}

static bool qtype_ok(int qt) { return qt == PI_QT_F32 || qt == PI_QT_Q4_0 || qt == PI_QT_Q8_0; }

#define ST(s) ((cudaStream_t)(s))
#define LAUNCH_CHECK(what) \
    if (pi_cuda_check(ctx, cudaGetLastError(), what)) return PI_ERR_CUDA

static unsigned nblocks(int64_t n, int thr) { return (unsigned)((n + thr - 1) / thr); }

extern "C" int pi_dequantize(pi_ctx* ctx, const void* raw, uint64_t raw_len, int qtype, int64_t rows, int64_t cols,
                             float* out, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (!raw || !out || rows < 0 || cols < 0) return pi_set_error(ctx, PI_ERR_ARG, "dequantize: bad argument");
    if (!(qtype_ok(qtype) || qtype == PI_QT_F16)) return pi_set_error(ctx, PI_ERR_ARG, "dequantize: unsupported type");
    int64_t n = rows * cols;
    if (qtype == PI_QT_Q4_0 || qtype == PI_QT_Q8_0) n = rows * (cols / 32) * 32;
    if ((int64_t)raw_len < gguf_size(qtype, n))
        return pi_set_error(ctx, PI_ERR_SHORT, "Insufficient data for dequantization");
    if (n == 0) return PI_OK;
    k_dequant<<<nblocks(n, 256), 256, 0, ST(stream)>>>((const uint8_t*)raw, qtype, n, out);
    LAUNCH_CHECK("dequantize");
    return PI_OK;
}

extern "C" int pi_quantize_q8_0(pi_ctx* ctx, const float* x, int64_t n, void* out_raw, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (!x || !out_raw || n < 0 || n % 32) return pi_set_error(ctx, PI_ERR_ARG, "quantize_q8_0: n % 32 != 0");
    if (n == 0) return PI_OK;
    k_quant_q8_blocks<<<nblocks(n, 256), 256, 0, ST(stream)>>>(x, n / 32, (uint8_t*)out_raw);
    LAUNCH_CHECK("quantize_q8_0");
    return PI_OK;
}

extern "C" int pi_quantize_q4_0(pi_ctx* ctx, const float* x, int64_t n, void* out_raw, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (!x || !out_raw || n < 0 || n % 32) return pi_set_error(ctx, PI_ERR_ARG, "quantize_q4_0: n % 32 != 0");
    if (n == 0) return PI_OK;
    k_quant_q4_blocks<<<nblocks(n, 256), 256, 0, ST(stream)>>>(x, n / 32, (uint8_t*)out_raw);
    LAUNCH_CHECK("quantize_q4_0");
    return PI_OK;
}

// rows of a col-major matvec, selected (idx) or all (idx == null, n_rows = n_out)
static int run_rows(pi_ctx* ctx, float* y, const float* x, const void* raw, int qtype, int64_t n_in, int64_t n_out,
                    const int64_t* idx, int64_t n_rows, cudaStream_t st) {
    if (n_rows == 0) return PI_OK;
    if (qtype == PI_QT_Q8_0 && n_in % 32 == 0) {
        char* scr;
        int rc = pi_scratch(ctx, st, (size_t)n_in + (size_t)(n_in / 32) * 4 + 512, &scr);
        if (rc) return rc;
        PiBump b{scr};
        int8_t* xq = b.take<int8_t>(n_in);
        float* xs = b.take<float>(n_in / 32);
        k_quant_act<<<nblocks(n_in, 256), 256, 0, st>>>(x, n_in, xq, xs);
        const size_t smem = (size_t)8 * (n_in / 32) * 4;
        if (smem > 200 * 1024) return pi_set_error(ctx, PI_ERR_ARG, "matvec: n_in too large");
        pi_smem_attr((const void*)k_rows_q8, smem);
        k_rows_q8<<<nblocks(n_rows, 8), 256, smem, st>>>(y, xq, xs, (const uint8_t*)raw, n_in, n_out, idx, n_rows,
                                                         ctx->dev_err);
    } else {
        k_rows_f32<<<nblocks(n_rows, 128), 128, 0, st>>>(y, x, (const uint8_t*)raw, qtype, n_in, n_out, idx, n_rows,
                                                          ctx->dev_err);
    }
    LAUNCH_CHECK("matvec");
    return PI_OK;
}

static int check_mv(pi_ctx* ctx, int qtype, int64_t n_in, int64_t n_out) {
    if (!qtype_ok(qtype)) return pi_set_error(ctx, PI_ERR_ARG, "unsupported quantisation type");
    if (n_in < 0 || n_out < 0) return pi_set_error(ctx, PI_ERR_ARG, "negative size");
    if (qtype != PI_QT_F32 && n_in % 32) return pi_set_error(ctx, PI_ERR_ARG, "n_in must be a multiple of 32");
    return PI_OK;
}

extern "C" int pi_matvec_col_major(pi_ctx* ctx, float* y, const float* x, const void* raw, int qtype, int64_t n_in,
                                   int64_t n_out, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (int rc = check_mv(ctx, qtype, n_in, n_out)) return rc;
    return run_rows(ctx, y, x, raw, qtype, n_in, n_out, nullptr, n_out, ST(stream));
}

extern "C" int pi_matvec_col_major_select(pi_ctx* ctx, float* y, const float* x, const void* raw, int qtype,
                                          int64_t n_in, int64_t n_out, const int64_t* idx, int64_t n_idx,
                                          void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (int rc = check_mv(ctx, qtype, n_in, n_out)) return rc;
    if (n_idx > 0 && !idx) return pi_set_error(ctx, PI_ERR_ARG, "null index list");
    return run_rows(ctx, y, x, raw, qtype, n_in, n_out, idx, n_idx, ST(stream));
}

extern "C" int pi_matvec_col_major_sparse_input(pi_ctx* ctx, float* y, const float* x, const int64_t* idx,
                                                int64_t n_idx, const void* raw, int qtype, int64_t n_in,
                                                int64_t n_out, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (int rc = check_mv(ctx, qtype, n_in, n_out)) return rc;
    if (n_out == 0) return PI_OK;
    if (n_idx == 0) {
        if (pi_cuda_check(ctx, cudaMemsetAsync(y, 0, sizeof(float) * n_out, ST(stream)), "memset")) return PI_ERR_CUDA;
        return PI_OK;
    }
    k_sparse_input<<<nblocks(n_out, 128), 128, 0, ST(stream)>>>(y, x, idx, n_idx, (const uint8_t*)raw, qtype, n_in,
                                                                 n_out, ctx->dev_err);
    LAUNCH_CHECK("sparse_input");
    return PI_OK;
}

static int ffn_core(pi_ctx* ctx, float* out, const float* x, const void* g, const void* u, const void* dn, int qtype,
                    int64_t n_embd, int64_t n_ff, const int64_t* idx, int64_t n_sel, cudaStream_t st) {
    // scratch: gate/up [n_sel] f32, plus the Q8_0 quantised hidden for dense down
    char* scr;
    const size_t need = (size_t)n_sel * 8 + 1024 + (size_t)n_ff + (size_t)n_ff / 8 + (size_t)n_embd + n_embd / 8 + 2048;
    int rc = pi_scratch(ctx, st, need, &scr);
    if (rc) return rc;
    PiBump b{scr};
    float* gv = b.take<float>(n_sel);
    float* uv = b.take<float>(n_sel);
    // the row kernels use the arena tail for the quantised x; give them their own offset
    (void)b;
    // run gate/up with row kernels that quantise x into a separate region
    if (qtype == PI_QT_Q8_0) {
        int8_t* xq = b.take<int8_t>(n_embd);
        float* xs = b.take<float>(n_embd / 32);
        k_quant_act<<<nblocks(n_embd, 256), 256, 0, st>>>(x, n_embd, xq, xs);
        const size_t smem = (size_t)8 * (n_embd / 32) * 4;
        pi_smem_attr((const void*)k_rows_q8, smem);
        k_rows_q8<<<nblocks(n_sel, 8), 256, smem, st>>>(gv, xq, xs, (const uint8_t*)g, n_embd, n_ff, idx, n_sel,
                                                        ctx->dev_err);
        k_rows_q8<<<nblocks(n_sel, 8), 256, smem, st>>>(uv, xq, xs, (const uint8_t*)u, n_embd, n_ff, idx, n_sel,
                                                        ctx->dev_err);
    } else {
        k_rows_f32<<<nblocks(n_sel, 128), 128, 0, st>>>(gv, x, (const uint8_t*)g, qtype, n_embd, n_ff, idx, n_sel,
                                                         ctx->dev_err);
        k_rows_f32<<<nblocks(n_sel, 128), 128, 0, st>>>(uv, x, (const uint8_t*)u, qtype, n_embd, n_ff, idx, n_sel,
                                                         ctx->dev_err);
    }
    k_swiglu_vec<<<nblocks(n_sel, 256), 256, 0, st>>>(gv, uv, n_sel);
    if (idx) {
        // selected: down over the sparse input (x = h at rows idx), f32 h
        k_sparse_input<<<nblocks(n_embd, 128), 128, 0, st>>>(out, gv, idx, n_sel, (const uint8_t*)dn, qtype, n_ff,
                                                              n_embd, ctx->dev_err);
    } else if (qtype == PI_QT_Q8_0) {
        int8_t* hq = b.take<int8_t>(n_ff);
        float* hs = b.take<float>(n_ff / 32);
        k_quant_act<<<nblocks(n_ff, 256), 256, 0, st>>>(gv, n_ff, hq, hs);
        const size_t smem = (size_t)8 * (n_ff / 32) * 4;
        pi_smem_attr((const void*)k_rows_q8, smem);
        k_rows_q8<<<nblocks(n_embd, 8), 256, smem, st>>>(out, hq, hs, (const uint8_t*)dn, n_ff, n_embd, nullptr,
                                                         n_embd, ctx->dev_err);
    } else {
        k_rows_f32<<<nblocks(n_embd, 128), 128, 0, st>>>(out, gv, (const uint8_t*)dn, qtype, n_ff, n_embd, nullptr,
                                                          n_embd, ctx->dev_err);
    }
    LAUNCH_CHECK("ffn_swiglu_q");
    return PI_OK;
}

extern "C" int pi_ffn_swiglu_q(pi_ctx* ctx, float* out, const float* x, const void* gate_raw, const void* up_raw,
                               const void* down_raw, int qtype, int64_t n_embd, int64_t n_ff, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (int rc = check_mv(ctx, qtype, n_embd, n_ff)) return rc;
    if (qtype != PI_QT_F32 && n_ff % 32) return pi_set_error(ctx, PI_ERR_ARG, "n_ff must be a multiple of 32");
    return ffn_core(ctx, out, x, gate_raw, up_raw, down_raw, qtype, n_embd, n_ff, nullptr, n_ff, ST(stream));
}

extern "C" int pi_ffn_swiglu_q_selected(pi_ctx* ctx, float* out, const float* x, const void* gate_raw,
                                        const void* up_raw, const void* down_raw, int qtype, int64_t n_embd,
                                        int64_t n_ff, const int64_t* idx, int64_t n_idx, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (int rc = check_mv(ctx, qtype, n_embd, n_ff)) return rc;
    if (n_idx == 0) {
        if (pi_cuda_check(ctx, cudaMemsetAsync(out, 0, sizeof(float) * n_embd, ST(stream)), "memset"))
            return PI_ERR_CUDA;
        return PI_OK;
    }
    if (n_idx >= n_ff) return pi_ffn_swiglu_q(ctx, out, x, gate_raw, up_raw, down_raw, qtype, n_embd, n_ff, stream);
    if (!idx) return pi_set_error(ctx, PI_ERR_ARG, "null index list");
    return ffn_core(ctx, out, x, gate_raw, up_raw, down_raw, qtype, n_embd, n_ff, idx, n_idx, ST(stream));
}

extern "C" int pi_sparse_ffn_create(pi_ctx* ctx, const void* gate_raw, const void* up_raw, const void* down_raw,
                                    int32_t qtype, int64_t n_embd, int64_t n_ff, int32_t src_on_host,
                                    pi_sparse_ffn** out) {
    if (!ctx || !out) return PI_ERR_ARG;
    *out = nullptr;
    if (qtype != PI_QT_Q4_0 && qtype != PI_QT_Q8_0)
        return pi_set_error(ctx, PI_ERR_ARG, "sparse ffn: weights must be Q4_0 or Q8_0");
    const int64_t unit = qtype == PI_QT_Q4_0 ? 1024 : 512;
    if (n_embd % unit || n_embd / unit > 4 || n_embd / unit < 1 || n_ff % 64 || n_embd % 1024 || n_ff > SF_MAX_FF)
        return pi_set_error(ctx, PI_ERR_ARG,
                            "sparse ffn: n_embd must be 1024/2048/4096, n_ff % 64 == 0 and n_ff <= 131072");
    cudaSetDevice(ctx->device);
    pi_sparse_ffn* F = new pi_sparse_ffn();
    F->ctx = ctx;
    F->n_embd = n_embd;
    F->n_ff = n_ff;
    F->qtype = qtype;
    int rc = pi_repack_mats(ctx, &F->gate, gate_raw, qtype, 1, n_ff, n_embd, src_on_host, &F->allocs);
    if (!rc) rc = pi_repack_mats(ctx, &F->up, up_raw, qtype, 1, n_ff, n_embd, src_on_host, &F->allocs);
    const int64_t dbytes = gguf_size(qtype, n_embd * n_ff);
    const void* dsrc = down_raw;
    void* stage = nullptr;
    if (!rc && src_on_host) {
        if (pi_cuda_check(ctx, cudaMalloc(&stage, dbytes), "cudaMalloc")) rc = PI_ERR_OOM;
        else if (pi_cuda_check(ctx, cudaMemcpy(stage, down_raw, dbytes, cudaMemcpyHostToDevice), "upload"))
            rc = PI_ERR_CUDA;
        dsrc = stage;
    }
    if (!rc) {
        const int64_t qb = qtype == PI_QT_Q4_0 ? n_ff * n_embd / 2 : n_ff * n_embd;
        if (pi_cuda_check(ctx, cudaMalloc(&F->down_q, qb), "cudaMalloc")) rc = PI_ERR_OOM;
        else F->allocs.push_back(F->down_q);
        if (!rc && pi_cuda_check(ctx, cudaMalloc(&F->down_d, (n_ff / 32) * n_embd * 2), "cudaMalloc")) rc = PI_ERR_OOM;
        else if (!rc) F->allocs.push_back(F->down_d);
    }
    if (!rc) {
        // mask [n_ff] bytes, then the work list [n_ff] int32 and its two counters, the fused
        // pass's grid barrier and its per-range tickets [n_ff / 32]
        const size_t mb = (size_t)n_ff + (size_t)n_ff * 4 + 64 + 64 + (size_t)(n_ff / 32) * 4;
        if (pi_cuda_check(ctx, cudaMalloc(&F->mask, mb), "cudaMalloc")) rc = PI_ERR_OOM;
        else F->allocs.push_back(F->mask);
        if (!rc && pi_cuda_check(ctx, cudaMemset(F->mask, 0, mb), "memset")) rc = PI_ERR_CUDA;
        F->wlist = reinterpret_cast<int32_t*>(F->mask + n_ff);
        F->wctr = reinterpret_cast<uint32_t*>(F->wlist + n_ff);
        F->fbar = reinterpret_cast<uint32_t*>(F->mask + n_ff + n_ff * 4 + 64);
        F->tick = reinterpret_cast<uint32_t*>(F->mask + n_ff + n_ff * 4 + 128);
        const char* split = getenv("PI_SF_SPLIT");
        F->fused = !(split && split[0] == '1');
    }
    if (!rc) {
        const int64_t nthr = (n_embd / 2) * (n_ff / 32);
        k_repack_down_nm<<<nblocks(nthr, 256), 256>>>((const uint8_t*)dsrc, qtype, n_embd, n_ff,
                                                      (uint8_t*)F->down_q, F->down_d);
        if (pi_cuda_check(ctx, cudaDeviceSynchronize(), "repack down")) rc = PI_ERR_CUDA;
    }
    if (stage) cudaFree(stage);
    if (rc) {
        pi_sparse_ffn_destroy(F);
        return rc;
    }
    *out = F;
    return PI_OK;
}

extern "C" void pi_sparse_ffn_destroy(pi_sparse_ffn* F) {
    if (!F) return;
    for (void* p : F->allocs) cudaFree(p);
    delete F;
}

// One fused launch for a one-token pass (k_sf_fused): grid = one CTA per SM, all
// resident (its grid barrier needs that).
static int sf_forward_fused(pi_ctx* ctx, pi_sparse_ffn* F, const float* x, int64_t T, const int64_t* ptr,
                            const int64_t* idx, float* out, cudaStream_t st, float* hb, const int8_t* xq,
                            const float* xs, int sms) {
    const int64_t d = F->n_embd, n_ff = F->n_ff;
    const bool q4 = F->qtype == PI_QT_Q4_0;
    const int n_cc = (int)(d / 512);
    const int64_t groups = n_ff / 32, per = std::max(1, sms / n_cc);
    const int gpr = (int)std::min<int64_t>(SF_FMAXG, (groups + per - 1) / per);
    {
        const int64_t t0 = 0;
        const int nt = 1, ntm = 1;
        const size_t xst = q4 ? (size_t)nt * (d / 32) * 36 * 4 : (size_t)nt * d + (size_t)nt * (d / 32) * 4;
        // down chunks: at least 128 neurons, more where the gate/up staging leaves room
        const size_t perb = 2 * (size_t)(q4 ? 256 : 512) + 2 * (size_t)ntm * 4, red = (size_t)ntm * 256 * 8;
        const size_t stage = (std::max(xst, 128 * perb + red) + 15) & ~(size_t)15;
        const int fch = (int)std::min<size_t>(1024, (stage - red) / perb / 32 * 32);
        const size_t smem = stage + SF_FMAXG * 1024 + 1024 * 4;
        SfFusedArgs a;
        a.G = (const uint8_t*)F->gate.q;
        a.U = (const uint8_t*)F->up.q;
        a.GD = F->gate.d;
        a.UD = F->up.d;
        a.DQ = (const uint8_t*)F->down_q;
        a.DS = F->down_d;
        a.mask = F->mask;
        a.wlist = F->wlist;
        a.wctr = F->wctr;
        a.tick = F->tick;
        a.bar = reinterpret_cast<SfGridBar*>(F->fbar);
        a.x = x;
        a.xq = xq;
        a.xs = xs;
        a.ptr = ptr;
        a.idx = idx;
        a.t0 = (int)t0;
        a.nt = nt;
        a.rn = 32 * gpr;
        a.fch = fch;
        a.n_embd = d;
        a.n_ff = n_ff;
        a.h = hb;
        a.y = out;
        a.err = ctx->dev_err;
        a.stage_bytes = (uint32_t)stage;
        PiProfScope ps(ctx, st, "k_sf_fused");
#define SF_FU(QT, B)                                                                         \
    {                                                                                        \
        auto kf = k_sf_fused<QT, B>;                                                         \
        pi_smem_attr((const void*)kf, smem);                                                 \
        int occ = 0;                                                                         \
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kf, SF_FT, smem);                \
        if (occ < 1) return pi_set_error(ctx, PI_ERR_CUDA, "sparse ffn: fused pass does not fit an SM"); \
        pi_pdl_launch(kf, dim3((unsigned)sms), dim3(SF_FT), smem, st, a);                    \
    }
        switch ((q4 ? 1 : 16) * (int)(d / 1024)) {
            case 1: SF_FU(PI_QT_Q4_0, 1) break;
            case 2: SF_FU(PI_QT_Q4_0, 2) break;
            case 4: SF_FU(PI_QT_Q4_0, 4) break;
            case 16: SF_FU(PI_QT_Q8_0, 1) break;
            case 32: SF_FU(PI_QT_Q8_0, 2) break;
            case 64: SF_FU(PI_QT_Q8_0, 4) break;
            default: return pi_set_error(ctx, PI_ERR_ARG, "sparse ffn: n_embd must be 1024, 2048 or 4096");
        }
#undef SF_FU
        LAUNCH_CHECK("sparse ffn (fused)");
    }
    return PI_OK;
}

extern "C" int pi_sparse_ffn_forward(pi_ctx* ctx, pi_sparse_ffn* F, const float* x, int64_t T, const int64_t* ptr,
                                     const int64_t* idx, float* out, void* stream) {
    if (!ctx || !F) return PI_ERR_ARG;
    if (T < 0 || (T > 0 && (!x || !ptr || !out))) return pi_set_error(ctx, PI_ERR_ARG, "sparse ffn: bad argument");
    if (T == 0) return PI_OK;
    if (((uintptr_t)x | (uintptr_t)out) & 15) return pi_set_error(ctx, PI_ERR_ARG, "sparse ffn: x, out 16-byte aligned");
    cudaStream_t st = ST(stream);
    const int64_t d = F->n_embd, n_ff = F->n_ff;
    char* scr;
    const size_t need = (size_t)SF_TMAX * n_ff * 4 + (size_t)T * d + (size_t)T * (d / 32) * 4 + 4096;
    if (int rc = pi_scratch(ctx, st, need, &scr)) return rc;
    PiBump b{scr};
    float* hb = b.take<float>((size_t)SF_TMAX * n_ff);
    int8_t* xq = nullptr;
    float* xs = nullptr;
    const bool q4 = F->qtype == PI_QT_Q4_0;
    if (!q4) {
        xq = b.take<int8_t>(T * d);
        xs = b.take<float>(T * (d / 32));
        PiProfScope ps(ctx, st, "k_sf_quant");
        k_quant_act<<<nblocks(T * d, 256), 256, 0, st>>>(x, T * d, xq, xs);
    }
    const int sms = ctx->sm_count > 0 ? ctx->sm_count : 148;
    if (d != 1024 && d != 2048 && d != 4096) return pi_set_error(ctx, PI_ERR_ARG, "sparse ffn: n_embd must be 1024, 2048 or 4096");
    if (F->fused && T == 1) return sf_forward_fused(ctx, F, x, T, ptr, idx, out, st, hb, xq, xs, sms);
    for (int64_t t0 = 0; t0 < T; t0 += SF_TMAX) {
        const int nt = (int)std::min<int64_t>(SF_TMAX, T - t0);
        {
            PiProfScope ps(ctx, st, "k_sf_mark");
            pi_pdl_launch(k_sf_mark, dim3((unsigned)std::min<int64_t>(nt * n_ff / 1024 + 1, 512)), dim3(256), 0, st,
                ptr, idx, (int)t0, nt, n_ff, reinterpret_cast<uint32_t*>(F->mask), F->wlist, F->wctr, hb, ctx->dev_err);
        }
        {
            PiProfScope ps(ctx, st, "k_sf_gateup");
            const size_t smem = q4 ? (size_t)nt * (d / 32) * 36 * 4 : (size_t)nt * d + (size_t)nt * (d / 32) * 4;
            const uint8_t* G = (const uint8_t*)F->gate.q;
            const uint8_t* U = (const uint8_t*)F->up.q;
#define SF_GU(QT, B)                                                                                            \
    {                                                                                                           \
        if (nt == 1) {                                                                                          \
            pi_smem_attr((const void*)k_sf_gateup<QT, B, 1>, smem);                                             \
            pi_pdl_launch(k_sf_gateup<QT, B, 1>, dim3((unsigned)sms), dim3(SF_GU_WARPS * 32), smem, st,        \
                G, U, F->gate.d, F->up.d, F->mask, x, xq, xs, ptr, F->wlist, F->wctr, (int)t0, nt, n_ff, hb, out); \
        } else {                                                                                                \
            pi_smem_attr((const void*)k_sf_gateup<QT, B, SF_TMAX>, smem);                                       \
            pi_pdl_launch(k_sf_gateup<QT, B, SF_TMAX>, dim3((unsigned)sms), dim3(SF_GU_WARPS * 32), smem, st,  \
                G, U, F->gate.d, F->up.d, F->mask, x, xq, xs, ptr, F->wlist, F->wctr, (int)t0, nt, n_ff, hb, out); \
        }                                                                                                       \
    }
            switch ((q4 ? 1 : 16) * (int)(d / 1024)) {
                case 1: SF_GU(PI_QT_Q4_0, 1) break;
                case 2: SF_GU(PI_QT_Q4_0, 2) break;
                case 4: SF_GU(PI_QT_Q4_0, 4) break;
                case 16: SF_GU(PI_QT_Q8_0, 1) break;
                case 32: SF_GU(PI_QT_Q8_0, 2) break;
                case 64: SF_GU(PI_QT_Q8_0, 4) break;
                default: return pi_set_error(ctx, PI_ERR_ARG, "sparse ffn: n_embd must be 1024, 2048 or 4096");
            }
#undef SF_GU
        }
        {
            PiProfScope ps(ctx, st, "k_sf_down");
            const dim3 dg((unsigned)(d / 512), (unsigned)((n_ff + SF_DN - 1) / SF_DN));
            const uint8_t* DQ = (const uint8_t*)F->down_q;
#define SF_DOWN(QT, NTM) pi_pdl_launch(k_sf_down<QT, NTM>, dg, dim3(256), 0, st, DQ, F->down_d, hb, ptr, (int)t0, nt, d, n_ff, out, F->wctr, F->mask)
            if (q4) {
                if (nt == 1) SF_DOWN(PI_QT_Q4_0, 1);
                else SF_DOWN(PI_QT_Q4_0, SF_TMAX);
            } else {
                if (nt == 1) SF_DOWN(PI_QT_Q8_0, 1);
                else SF_DOWN(PI_QT_Q8_0, SF_TMAX);
            }
#undef SF_DOWN
        }
        LAUNCH_CHECK("sparse ffn");
    }
    return PI_OK;
}

extern "C" int pi_predictor_forward(pi_ctx* ctx, const float* a, int64_t T, const float* W1, const float* b1,
                                    const float* W2, const float* b2, int64_t n_in, int64_t n_hidden, int64_t n_out,
                                    float* probs, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (T <= 0) return PI_OK;
    if (!a || !W1 || !b1 || !W2 || !b2 || !probs) return pi_set_error(ctx, PI_ERR_ARG, "predictor: null pointer");
    char* scr;
    if (int rc = pi_scratch(ctx, ST(stream), (size_t)T * n_hidden * 4 + 256, &scr)) return rc;
    float* h = reinterpret_cast<float*>(scr);
    k_pred_layer<<<dim3(nblocks(n_hidden, 128), (unsigned)T), 128, 0, ST(stream)>>>(a, T, n_in, W1, b1, n_hidden, 0, h);
    k_pred_layer<<<dim3(nblocks(n_out, 128), (unsigned)T), 128, 0, ST(stream)>>>(h, T, n_hidden, W2, b2, n_out, 1,
                                                                                 probs);
    LAUNCH_CHECK("predictor");
    return PI_OK;
}

// --------------------------------------------------------------------------
// Device hot-neuron lists for the sparse FFN (CSR: ptr [T+1], idx ascending per token).
//   from predictor probabilities: Predictor::predict_hot (predictor/mod.rs:87-95,
//   blocks with p >= threshold, ascending) with block b covering neurons
//   [b * block, (b + 1) * block) of n_ff (predictor/mod.rs:15: blocks of 64);
//   from a static list (a HotNeuronIndex layer, model/mod.rs:1743-1761): the same
//   list for every token.
// One CTA walks the tokens in order and keeps the running offset.
// --------------------------------------------------------------------------
__global__ __launch_bounds__(1024) void k_hot_from_probs(const float* __restrict__ probs, int T, int n_blocks,
                                                         float threshold, int block, int64_t n_ff,
                                                         int64_t* __restrict__ ptr, int64_t* __restrict__ idx) {
    __shared__ int64_t s_scan[1024];
    __shared__ int64_t s_base;
    if (threadIdx.x == 0) {
        s_base = 0;
        ptr[0] = 0;
    }
    __syncthreads();
    for (int t = 0; t < T; ++t) {
        for (int b0 = 0; b0 < n_blocks; b0 += 1024) {
            const int b = b0 + threadIdx.x;
            int64_t n = 0;
            if (b < n_blocks) {
                const float p = probs[(size_t)t * n_blocks + b];
                const int64_t lo = (int64_t)b * block, hi = min((int64_t)(b + 1) * block, n_ff);
                if (p >= threshold && lo < hi) n = hi - lo;
            }
            s_scan[threadIdx.x] = n;
            __syncthreads();
            for (int o = 1; o < 1024; o <<= 1) {  // inclusive scan of the blocks' neuron counts
                const int64_t v = threadIdx.x >= (unsigned)o ? s_scan[threadIdx.x - o] : 0;
                __syncthreads();
                s_scan[threadIdx.x] += v;
                __syncthreads();
            }
            const int64_t at = s_base + s_scan[threadIdx.x] - n;
            for (int64_t j = 0; j < n; ++j) idx[at + j] = (int64_t)b * block + j;
            __syncthreads();
            if (threadIdx.x == 0) s_base += s_scan[1023];
            __syncthreads();
        }
        if (threadIdx.x == 0) ptr[t + 1] = s_base;
    }
}

__global__ void k_hot_broadcast(const int64_t* __restrict__ list, int64_t n, int T, int64_t* __restrict__ ptr,
                                int64_t* __restrict__ idx) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i <= T) ptr[i] = i * n;
    if (i < (int64_t)T * n) idx[i] = list[i % n];
}

extern "C" int pi_hot_lists_from_probs(pi_ctx* ctx, const float* probs, int64_t T, int64_t n_blocks, float threshold,
                                       int64_t block, int64_t n_ff, int64_t* ptr, int64_t* idx, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (T < 0 || T > (1 << 20) || n_blocks < 1 || block < 1 || n_ff < 1 || !ptr || (T > 0 && (!probs || !idx)))
        return pi_set_error(ctx, PI_ERR_ARG, "hot lists: bad sizes or pointers");
    k_hot_from_probs<<<1, 1024, 0, ST(stream)>>>(probs, (int)T, (int)n_blocks, threshold, (int)block, n_ff, ptr, idx);
    LAUNCH_CHECK("hot lists");
    return PI_OK;
}

extern "C" int pi_hot_lists_broadcast(pi_ctx* ctx, const int64_t* list, int64_t n, int64_t T, int64_t* ptr,
                                      int64_t* idx, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (T < 0 || T > (1 << 20) || n < 0 || !ptr || (n > 0 && T > 0 && (!list || !idx)))
        return pi_set_error(ctx, PI_ERR_ARG, "hot lists: bad sizes or pointers");
    const int64_t m = std::max<int64_t>(T * n, T + 1);
    k_hot_broadcast<<<nblocks(m, 256), 256, 0, ST(stream)>>>(list, n, (int)T, ptr, idx);
    LAUNCH_CHECK("hot lists");
    return PI_OK;
}

extern "C" int pi_synth_normal(pi_ctx* ctx, uint64_t seed, uint64_t offset, int64_t n, float stdv, float* out,
                               void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (n <= 0) return PI_OK;
    k_synth<<<nblocks(n, 256), 256, 0, ST(stream)>>>(seed, offset, n, stdv, out);
    LAUNCH_CHECK("synth");
    return PI_OK;
}

extern "C" int pi_synth_normal_host(uint64_t seed, uint64_t offset, int64_t n, float stdv, float* out) {
    for (int64_t k = 0; k < n; ++k) {
        const uint64_t i = offset + (uint64_t)k, m = i >> 1;
        const double u1 = 1.0 - (double)(splitmix_at(seed, 2 * m) >> 11) * (1.0 / 9007199254740992.0);
        const double u2 = (double)(splitmix_at(seed, 2 * m + 1) >> 11) * (1.0 / 9007199254740992.0);
        const double r = std::sqrt(-2.0 * std::log(u1));
        const double th = 6.283185307179586 * u2;
        const double v = (i & 1) ? r * std::sin(th) : r * std::cos(th);
        out[k] = (float)(v * (double)stdv);
    }
    return PI_OK;
}

// ===========================================================================
// Allocation-free Q8_0 matvec.
//
// pi_matvec_col_major quantises x into scratch that its context allocates on
// first use. Some hosts cannot allocate device memory at the point of the
// call: an embedding whose allocator forbids cudaMalloc on its hot path (for
// example a runtime that preallocates all device memory up front, or a
// process that drives the GPU under a stream capture it does not own). For
// them the variant below keeps its scratch -- the quantised copy of x -- in a
// fixed file-scope device array, so the call allocates nothing and needs no
// pi_ctx. Every GPU that loads this library reserves the array until exit.
// ===========================================================================
#include <mutex>

namespace {
constexpr int64_t PI_STATIC_MAX_N_IN = 16384;  // largest n_in the fixed scratch holds
struct StaticScratch {
    int8_t xq[PI_STATIC_MAX_N_IN];
    float xs[PI_STATIC_MAX_N_IN / 32];
};
static __device__ __align__(256) StaticScratch g_static_scratch;

// Device addresses of g_static_scratch, looked up once per device (the host
// symbol is only a stand-in and must never be handed to a kernel).
constexpr int PI_MAX_DEVICES = 64;
std::mutex g_static_mu;
StaticScratch* g_static_ptr[PI_MAX_DEVICES] = {};
}  // namespace

extern "C" int pi_matvec_col_major_q8_0_noalloc(float* y, const float* x, const void* raw, int64_t n_in,
                                                int64_t n_out, void* stream) {
    if (!y || !x || !raw || n_in <= 0 || n_out < 0 || n_in % 32) return PI_ERR_ARG;
    if (n_in > PI_STATIC_MAX_N_IN) return PI_ERR_ARG;  // beyond the fixed scratch
    if (n_out == 0) return PI_OK;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= PI_MAX_DEVICES) {
        cudaGetLastError();
        return PI_ERR_CUDA;
    }
    StaticScratch* scr;
    {
        std::lock_guard<std::mutex> g(g_static_mu);
        if (!g_static_ptr[dev]) {
            void* p = nullptr;
            if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) {
                cudaGetLastError();
                return PI_ERR_CUDA;
            }
            g_static_ptr[dev] = static_cast<StaticScratch*>(p);
        }
        scr = g_static_ptr[dev];
    }
    cudaStream_t st = (cudaStream_t)stream;
    // k_quant_act writes every byte of xq[0, n_in) and xs[0, n_in/32) before
    // k_rows_q8 reads them, so nothing left by an earlier call is read.
    k_quant_act<<<nblocks(n_in, 256), 256, 0, st>>>(x, n_in, scr->xq, scr->xs);
    const size_t smem = (size_t)8 * (n_in / 32) * 4;  // <= 16 KiB for n_in <= 16384
    k_rows_q8<<<nblocks(n_out, 8), 256, smem, st>>>(y, scr->xq, scr->xs, (const uint8_t*)raw, n_in, n_out, nullptr,
                                                    n_out, nullptr);
    return cudaGetLastError() == cudaSuccess ? PI_OK : PI_ERR_CUDA;
}
