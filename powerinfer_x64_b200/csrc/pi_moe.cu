// MoE feed-forward layer on B200: routing, dispatch, expert SwiGLU, combine.
//
// Reference path being replaced: model/mod.rs:1245-1571 (one token at a
// time, two CPU threads of quant::ffn_swiglu_q calls). Here one call runs a
// whole batch of T tokens through a few kernels on one stream:
//
//   k_prep        RMSNorm (optional, ops.rs:13-27 lane order) + Q8_0
//                 activation quantiser (quant/mod.rs:698-736), per token.
//   routing       router logits in the reference's sequential f32 order
//                 (quant/mod.rs:921-935), row E = the shared-expert gate
//                 (model/mod.rs:1500-1509), then softmax -> top-k (ties to the
//                 lowest index) -> ascending sort -> renormalised gates
//                 (model/mod.rs:1278-1312):
//                   decode    k_router_dec (one exact chain per lane; for T <= 8
//                             it also runs the top-k) + k_topk;
//                   prefill   tensor-core logits certified by an error bound
//                             (pi_prefill.cu) + k_router_cand, exact chains for
//                             the uncertain tokens (k_router_exact_list);
//                             k_router_wide when forced or E > 256.
//   k_dispatch    per-expert counts, offsets, stable token permutation and
//                 the work-item list for the expert kernels (no reference
//                 counterpart: the reference loops token by token).
//   experts       decode: k_gateup_* (gate+up GEMV, SwiGLU), k_quant_h (Q8_0
//                 re-quantisation of h, quant/mod.rs:1179-1204), k_down_q8s /
//                 k_down_q4; prefill: the tcgen05 GEMMs of pi_prefill.cu and
//                 pi_prefill_q8.cu.
//   k_combine     ascending-expert gate-weighted sum + sigmoid-gated shared
//                 expert + optional residual (model/mod.rs:1525-1534,
//                 :1627-1633), in the reference's exact f32 order.
//
// The decode expert kernels stream each weight row from HBM once per work item
// with 16-byte coalesced loads (gate/up into registers, down through a bulk-copy
// ring in shared memory) and loop over the item's tokens: HBM-bound.
#include "pi_tc.cuh"
// pi_tc.cuh (pi_common.cuh) comes first: it names the quant types that pi_moe.h defines as macros
#include "pi_internal.h"

#include <algorithm>
#include <cstdlib>

namespace {

constexpr int TG = 16;  // tokens per work item (gate/up quantises h with one warp per token)

// One token row xr (global or shared memory) by an NT-thread CTA; __syncthreads inside.
template <int NT = 256>
PI_DEV void split_row(const float* xr, int t, int d, __half* __restrict__ xh, __half* __restrict__ xl,
                      float* __restrict__ xnorm) {
    __shared__ double red[NT / 32];
    __shared__ int s_bad;
    const int tid = threadIdx.x;
    if (tid == 0) s_bad = 0;
    __syncthreads();
    double ss = 0.0;
    bool bad = false;
    for (int c = tid * 8; c < d; c += NT * 8) {
        const float4 v0 = *reinterpret_cast<const float4*>(xr + c);
        const float4 v1 = *reinterpret_cast<const float4*>(xr + c + 4);
        const float f[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const __half2 hv = __floats2half2_rn(f[2 * q], f[2 * q + 1]);
            const float2 hf = __half22float2(hv);
            const __half2 lv = __floats2half2_rn(f[2 * q] - hf.x, f[2 * q + 1] - hf.y);
            hi[q] = *reinterpret_cast<const uint32_t*>(&hv);
            lo[q] = *reinterpret_cast<const uint32_t*>(&lv);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            ss += (double)f[j] * (double)f[j];
            bad |= !(fabsf(f[j]) < 32768.0f);
        }
        *reinterpret_cast<uint4*>(xh + (size_t)t * d + c) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(xl + (size_t)t * d + c) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    if (bad) s_bad = 1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
        double tot = 0.0;
        for (int w = 0; w < NT / 32; ++w) tot += red[w];
        // the f64 sum is within ~2^-40 relative; 1 + 2^-20 covers it and the f32 rounding
        xnorm[t] = s_bad ? INFINITY : __double2float_ru(__dsqrt_ru(tot) * (1.0 + 0x1p-20));
    }
}

// ---------------------------------------------------------------------------
// k_prep: optional RMSNorm, then Q8_0 quantisation of the (normed) tokens.
// grid T, block 256, dynamic shared memory d floats: the CTA stages its token
// row, four lanes run the reference's four sum-of-squares chains once, then
// every warp normalises and quantises 32-element blocks (one block per warp
// per pass).
// ---------------------------------------------------------------------------
// NT threads per token: 256 for a few tokens, 128 for large batches (more tokens per SM
// in flight while four lanes of each run the sequential sum of squares).
template <int NT>
__global__ __launch_bounds__(NT) void k_prep(const float* __restrict__ x, int d, int do_norm, float eps,
                                              float* __restrict__ normed, int do_quant, int8_t* __restrict__ xq,
                                              float* __restrict__ xs, __half* __restrict__ xh,
                                              __half* __restrict__ xl, float* __restrict__ xnorm) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    extern __shared__ float s_row[];
    __shared__ float s_inv;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float* xr = x + (size_t)t * d;
    for (int c = tid; c < d / 4; c += NT)
        *reinterpret_cast<float4*>(&s_row[4 * c]) = *reinterpret_cast<const float4*>(xr + 4 * c);
    __syncthreads();
    float inv = 1.0f;
    if (do_norm) {
        // sum_squares_sse (simd.rs:116-137): 4 lane accumulators over
        // elements i = 4m + lane, then (l0 + l1) + (l2 + l3), then a scalar tail.
        if (tid < 32) {
            const int lane = tid;
            float acc = 0.0f;
            const int n4 = d & ~3;
            if (lane < 4)
#pragma unroll 8
                for (int j = lane; j < n4; j += 4) acc = fadd(acc, fmul(s_row[j], s_row[j]));
            const float a1 = __shfl_sync(0xffffffffu, acc, 1);
            const float a2 = __shfl_sync(0xffffffffu, acc, 2);
            const float a3 = __shfl_sync(0xffffffffu, acc, 3);
            if (lane == 0) {
                float ss = fadd(fadd(acc, a1), fadd(a2, a3));
                for (int j = n4; j < d; ++j) ss = fadd(ss, fmul(s_row[j], s_row[j]));
                const float rms = __fsqrt_rn(fadd(fdiv(ss, (float)d), eps));
                s_inv = fdiv(1.0f, rms);
            }
        }
        __syncthreads();
        inv = s_inv;
    }
    // four consecutive elements per thread (d % 128 == 0, so every warp pass is full): eight
    // lanes hold one Q8_0 block, so its absmax takes three shuffles and its two divisions are
    // paid once per four elements (quad_quant_q8; quant/mod.rs:698-736)
    for (int c = tid; c < d / 4; c += NT) {
        float4 v = *reinterpret_cast<const float4*>(&s_row[4 * c]);
        if (do_norm) {
            v = make_float4(fmul(v.x, inv), fmul(v.y, inv), fmul(v.z, inv), fmul(v.w, inv));  // * weight (1.0)
            *reinterpret_cast<float4*>(normed + (size_t)t * d + 4 * c) = v;
            *reinterpret_cast<float4*>(&s_row[4 * c]) = v;
        }
        if (do_quant) {
            const float e[4] = {v.x, v.y, v.z, v.w};
            float sc;
            *reinterpret_cast<uint32_t*>(xq + (size_t)t * d + 4 * c) = quad_quant_q8(e, &sc);
            if ((c & 7) == 0) xs[(size_t)t * (d / 32) + c / 8] = sc;
        }
    }
    // the certified tensor-core router's f16 hi/lo split and norm bound of the (normed) row
    if (xh) split_row<NT>(s_row, t, d, xh, xl, xnorm);
}

// ---------------------------------------------------------------------------
// k_router: exact logits. Thread = expert row (E routed rows + row E for the
// shared-expert gate), TT tokens per CTA, each chain a sequential f32 sum in
// the reference's order: sum = sum + w[i] * x[i], i ascending, no FMA.
// grid (ceil((E+1)/128), ceil(T/TT)), block 128.
// ---------------------------------------------------------------------------
constexpr int RT_TT = 8, RT_CH = 256;
__global__ __launch_bounds__(128) void k_router(const float* __restrict__ xin, const float* __restrict__ W,
                                                const float* __restrict__ bias, int T, int d, int E, int nrows,
                                                float* __restrict__ logits) {
    __shared__ __align__(16) float xs[RT_TT][RT_CH];
    const int Ep1 = E + 1;
    const int e = blockIdx.x * 128 + threadIdx.x;
    const int t0 = blockIdx.y * RT_TT;
    const int nt = min(RT_TT, T - t0);
    const float* wr = W + (size_t)min(e, nrows - 1) * d;
    float acc[RT_TT];
#pragma unroll
    for (int t = 0; t < RT_TT; ++t) acc[t] = 0.0f;
    for (int c0 = 0; c0 < d; c0 += RT_CH) {
        __syncthreads();
        for (int q = threadIdx.x; q < RT_TT * RT_CH; q += 128) {
            int t = q / RT_CH, i = q % RT_CH;
            xs[t][i] = (t < nt && c0 + i < d) ? xin[(size_t)(t0 + t) * d + c0 + i] : 0.0f;
        }
        __syncthreads();
        const int lim = min(RT_CH, d - c0);
        for (int i = 0; i < lim; i += 4) {
            float4 w = __ldg(reinterpret_cast<const float4*>(wr + c0 + i));
#pragma unroll
            for (int t = 0; t < RT_TT; ++t) {
                float4 xv = *reinterpret_cast<const float4*>(&xs[t][i]);
                float a = acc[t];
                a = fadd(a, fmul(w.x, xv.x));
                a = fadd(a, fmul(w.y, xv.y));
                a = fadd(a, fmul(w.z, xv.z));
                a = fadd(a, fmul(w.w, xv.w));
                acc[t] = a;
            }
        }
    }
    if (e >= nrows) return;
#pragma unroll
    for (int t = 0; t < RT_TT; ++t) {
        if (t < nt) {
            float v = acc[t];
            if (bias && e < E) v = fadd(v, bias[e]);
            logits[(size_t)(t0 + t) * Ep1 + e] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// k_router_wide: exact logits of the E expert rows for prefill-sized batches.
// Each logit is the reference's sequential f32 sum (quant/mod.rs:921-935): the
// accumulator walks i in ascending order, one rounded mul then one rounded add
// per step (no FMA), bit for bit; with T x E independent chains the throughput,
// not the chain latency, sets the time.
// CTA = 32 tokens x 128 rows, 4 warps; warp w owns tokens 8w..8w+7, lane l rows
// 4l..4l+3 (32 accumulators). Per i a warp reads its 128 router values with one
// 16-byte shared load (router transposed to [d][ep], so the staging is
// coalesced) and its 8 token values with two broadcast loads. The next
// 32-i block is loaded into registers while the current one is consumed.
// ---------------------------------------------------------------------------
constexpr int RW_ROWS = 128, RW_K = 32, RW_THREADS = 128;
template <int TPW>  // tokens per warp
__global__ __launch_bounds__(RW_THREADS) void k_router_wide(const float* __restrict__ xin, const float* __restrict__ Wt,
                                                            int64_t ep, const float* __restrict__ bias,
                                                            const float* __restrict__ wgate, int T, int d, int E,
                                                            float* __restrict__ logits) {
    constexpr int RW_TOK = 4 * TPW, RW_XS = RW_TOK + 4, XV = RW_TOK * RW_K / 4 / RW_THREADS;
    __shared__ __align__(16) float ws[RW_K][RW_ROWS];
    __shared__ __align__(16) float xs[RW_K][RW_XS];  // [i][token]
    __shared__ __align__(16) float gs[RW_K];         // router row E (shared-expert gate)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * RW_TOK, e0 = blockIdx.y * RW_ROWS;
    // the CTAs of row block 0 also run the gate row's chain: lane l < TPW of warp
    // w for token TPW w + l
    const bool gate = wgate != nullptr && blockIdx.y == 0;
    float acc_g = 0.0f;
    float4 gr = make_float4(0.f, 0.f, 0.f, 0.f);
    float acc[TPW][4];
#pragma unroll
    for (int a = 0; a < TPW; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.0f;
    float4 wr[8], xr[XV];
    auto load = [&](int k0) {
        if (gate && tid < RW_K / 4) gr = __ldg(reinterpret_cast<const float4*>(wgate + k0 + 4 * tid));
#pragma unroll
        for (int m = 0; m < 8; ++m) {  // [32 i][128 rows]: a warp reads one i-row of 512 bytes
            const int q = tid + RW_THREADS * m, i = q >> 5, c4 = q & 31;
            wr[m] = __ldg(reinterpret_cast<const float4*>(Wt + (size_t)(k0 + i) * ep + e0 + 4 * c4));
        }
#pragma unroll
        for (int m = 0; m < XV; ++m) {  // [RW_TOK tokens][32 i]
            const int q = tid + RW_THREADS * m, tk = q >> 3, c4 = q & 7;
            xr[m] = (t0 + tk < T) ? *reinterpret_cast<const float4*>(xin + (size_t)(t0 + tk) * d + k0 + 4 * c4)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    load(0);
    for (int k0 = 0; k0 < d; k0 += RW_K) {
        __syncthreads();
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int q = tid + RW_THREADS * m;
            *reinterpret_cast<float4*>(&ws[q >> 5][4 * (q & 31)]) = wr[m];
        }
#pragma unroll
        for (int m = 0; m < XV; ++m) {
            const int q = tid + RW_THREADS * m, tk = q >> 3, i = 4 * (q & 7);
            xs[i][tk] = xr[m].x;
            xs[i + 1][tk] = xr[m].y;
            xs[i + 2][tk] = xr[m].z;
            xs[i + 3][tk] = xr[m].w;
        }
        if (gate && tid < RW_K / 4) *reinterpret_cast<float4*>(&gs[4 * tid]) = gr;
        __syncthreads();
        if (k0 + RW_K < d) load(k0 + RW_K);
        if (gate) {
#pragma unroll 8
            for (int i = 0; i < RW_K; ++i) acc_g = fadd(acc_g, fmul(gs[i], xs[i][TPW * warp + (lane % TPW)]));
        }
#pragma unroll 8
        for (int i = 0; i < RW_K; ++i) {
            const float4 wv = *reinterpret_cast<const float4*>(&ws[i][4 * lane]);
            float x8[TPW];
#pragma unroll
            for (int v = 0; v < TPW / 4; ++v) {
                const float4 xv = *reinterpret_cast<const float4*>(&xs[i][TPW * warp + 4 * v]);
                x8[4 * v] = xv.x; x8[4 * v + 1] = xv.y; x8[4 * v + 2] = xv.z; x8[4 * v + 3] = xv.w;
            }
            const float w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int a = 0; a < TPW; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = fadd(acc[a][b], fmul(w4[b], x8[a]));
        }
    }
#pragma unroll
    for (int a = 0; a < TPW; ++a) {
        const int t = t0 + TPW * warp + a;
        if (t >= T) continue;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int e = e0 + 4 * lane + b;
            if (e >= E) continue;
            float v = acc[a][b];
            if (bias) v = fadd(v, bias[e]);
            logits[(size_t)t * (E + 1) + e] = v;
        }
    }
    if (gate && lane < TPW && t0 + TPW * warp + lane < T) logits[(size_t)(t0 + TPW * warp + lane) * (E + 1) + E] = acc_g;
}

__global__ void k_transpose_rows(const float* __restrict__ src, int rows, int cols, int64_t ld_dst,
                                 float* __restrict__ dst) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * cols) return;
    const int r = (int)(i / cols), c = (int)(i % cols);
    dst[(size_t)c * ld_dst + r] = src[i];
}

// ---------------------------------------------------------------------------
// k_router_exact_list: exact (reference-order) logits for the tokens listed
// in list[0 .. *n_list). CTA = 32 router rows x one listed token at a time;
// the 256 threads stage 32 x 256 tiles of the rows in shared memory (next
// tile prefetched into registers), warp 0 runs one sequential chain per row
// (d must be a multiple of 256). grid (ceil((E+1)/32), G), block 256.
// ---------------------------------------------------------------------------
constexpr int EX_CH = 256, EX_THREADS = 256;
constexpr size_t EX_SMEM = (size_t)2 * 32 * (EX_CH + 1) * 4 + (size_t)2 * EX_CH * 4;
__global__ __launch_bounds__(EX_THREADS) void k_router_exact_list(const float* __restrict__ xin, const float* __restrict__ W,
                                                           const float* __restrict__ bias, int d, int E,
                                                           const int32_t* __restrict__ list,
                                                           const int32_t* __restrict__ n_list,
                                                           float* __restrict__ logits) {
    extern __shared__ float ex_sm[];
    float(*ws)[32][EX_CH + 1] = reinterpret_cast<float(*)[32][EX_CH + 1]>(ex_sm);
    float(*xs)[EX_CH] = reinterpret_cast<float(*)[EX_CH]>(ex_sm + 2 * 32 * (EX_CH + 1));
    const int n = *n_list;
    const int row0 = blockIdx.x * 32;
    const int nrow = min(32, E + 1 - row0);
    const int tid = threadIdx.x;
    const int ntiles = d / EX_CH;
    for (int g = blockIdx.y; g < n; g += gridDim.y) {
        const int t = list[g];
        const float* xr = xin + (size_t)t * d;
        float4 rw[8];
        float rx;
        auto load = [&](int tile) {
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int idx = tid + EX_THREADS * m;  // 2048 float4 = 32 rows x 64
                const int r = idx >> 6, j = idx & 63;
                rw[m] = (r < nrow) ? __ldg(reinterpret_cast<const float4*>(W + (size_t)(row0 + r) * d + tile * EX_CH) + j)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            rx = xr[tile * EX_CH + tid];
        };
        auto store = [&](int buf) {
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int idx = tid + EX_THREADS * m;
                const int r = idx >> 6, j = idx & 63;
                ws[buf][r][4 * j] = rw[m].x;
                ws[buf][r][4 * j + 1] = rw[m].y;
                ws[buf][r][4 * j + 2] = rw[m].z;
                ws[buf][r][4 * j + 3] = rw[m].w;
            }
            xs[buf][tid] = rx;
        };
        __syncthreads();
        load(0);
        store(0);
        __syncthreads();
        float acc = 0.0f;
        for (int tile = 0; tile < ntiles; ++tile) {
            const int buf = tile & 1;
            if (tile + 1 < ntiles) load(tile + 1);
            if (tid < nrow) {
                const float* wrow = ws[buf][tid];
                const float* xv = xs[buf];
#pragma unroll 32
                for (int i = 0; i < EX_CH; ++i) acc = fadd(acc, fmul(wrow[i], xv[i]));
            }
            if (tile + 1 < ntiles) store(buf ^ 1);
            __syncthreads();
        }
        if (tid < nrow) {
            const int e = row0 + tid;
            float v = acc;
            if (bias && e < E) v = fadd(v, bias[e]);
            logits[(size_t)t * (E + 1) + e] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// k_topk: one warp per token, NPL = ceil(E / 32) experts per lane.
// ---------------------------------------------------------------------------
constexpr int TK_WARPS = 4, TK_PER_LANE = 16;  // E <= 32 * TK_PER_LANE
// Routes every token from its exact logits, or (list != null) the listed tokens.
// Top-k by probability with ties to the lowest expert index: a round takes the
// largest key with redux.sync max (keys: probability bits + 2, order-preserving
// for non-negative floats; 1 for NaN, 0 for taken) and then the lowest index
// holding it with redux.sync min.
template <int NPL>
PI_DEV void topk_token(const float* __restrict__ logits, int t, int E, int k, int has_shgate,
                       int32_t* __restrict__ idx, float* __restrict__ gates, float* __restrict__ shscale,
                       int32_t* __restrict__ counts, float* p, int* sel, int lane) {
    const float* lr = logits + (size_t)t * (E + 1);
    float l[NPL];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        const int e = lane + 32 * j;
        l[j] = (e < E) ? __ldcg(lr + e) : -INFINITY;
        if (e < E) m = fmaxf(m, l[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        const int e = lane + 32 * j;
        if (e < E) p[e] = exp_cr(fsub(l[j], m));
    }
    __syncwarp();
    // exp_sum: sequential sum in expert order (model/mod.rs:1282)
    float es = 0.0f;
    if (lane == 0) {
#pragma unroll 16
        for (int e = 0; e < E; ++e) es = fadd(es, p[e]);
    }
    es = __shfl_sync(0xffffffffu, es, 0);
    float pr[NPL];
    uint32_t key[NPL];
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        const int e = lane + 32 * j;
        pr[j] = (e < E) ? fdiv(p[e], es) : 0.0f;
        key[j] = (e < E) ? (pr[j] == pr[j] ? __float_as_uint(pr[j]) + 2u : 1u) : 0u;
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        const int e = lane + 32 * j;
        if (e < E) p[e] = pr[j];
    }
    for (int r = 0; r < k; ++r) {
        uint32_t mk = 0;
#pragma unroll
        for (int j = 0; j < NPL; ++j) mk = max(mk, key[j]);
        mk = __reduce_max_sync(0xffffffffu, mk);
        uint32_t me = 0xffffffffu;
#pragma unroll
        for (int j = NPL - 1; j >= 0; --j)
            if (key[j] == mk) me = lane + 32 * j;
        const int bi = (int)__reduce_min_sync(0xffffffffu, me);
        if ((bi & 31) == lane) {
#pragma unroll
            for (int j = 0; j < NPL; ++j)
                if (j == (bi >> 5)) key[j] = 0;
        }
        if (lane == 0) sel[r] = bi;
    }
    __syncwarp();
    // ascending sort of the k selected indices (model/mod.rs:1303)
    const int mine = (lane < k) ? sel[lane] : 0x7fffffff;
    int rank = 0;
    for (int r = 0; r < k; ++r) rank += (sel[r] < mine);
    __syncwarp();
    if (lane < k) sel[rank] = mine;
    __syncwarp();
    float ssum = 0.0f;
    if (lane == 0)
        for (int r = 0; r < k; ++r) ssum = fadd(ssum, p[sel[r]]);
    ssum = __shfl_sync(0xffffffffu, ssum, 0);
    if (lane < k) {
        const int e = sel[lane];
        const float pe = p[e];
        idx[(size_t)t * k + lane] = e;
        gates[(size_t)t * k + lane] = (ssum > 0.0f) ? fdiv(pe, ssum) : pe;
        atomicAdd(&counts[e], 1);
    }
    if (lane == 0 && shscale) shscale[t] = has_shgate ? sigmoid_ref(__ldcg(lr + E)) : 1.0f;
    __syncwarp();
}

template <int NPL>
__global__ __launch_bounds__(TK_WARPS * 32) void k_topk(const float* __restrict__ logits, int T, int E, int k,
                                                        int has_shgate, int32_t* __restrict__ idx,
                                                        float* __restrict__ gates, float* __restrict__ shscale,
                                                        int32_t* __restrict__ counts,
                                                        const int32_t* __restrict__ list,
                                                        const int32_t* __restrict__ n_list) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    __shared__ float s_p[TK_WARPS][32 * NPL];
    __shared__ int s_sel[TK_WARPS][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tok = list ? *n_list : T;
    for (int g = blockIdx.x * TK_WARPS + warp; g < n_tok; g += gridDim.x * TK_WARPS)
        topk_token<NPL>(logits, list ? list[g] : g, E, k, has_shgate, idx, gates, shscale, counts, s_p[warp],
                        s_sel[warp], lane);
}

// k_topk for E experts (E <= 512).
void launch_topk(unsigned grid, cudaStream_t st, const float* logits, int T, int E, int k, int has_shgate,
                 int32_t* idx, float* gates, float* shscale, int32_t* counts, const int32_t* list,
                 const int32_t* n_list) {
#define TOPK(N) pi_pdl_launch(k_topk<N>, dim3(grid), dim3(TK_WARPS * 32), 0, st, logits, T, E, k, has_shgate, idx, gates, shscale, counts, list, n_list)
    if (E <= 64) TOPK(2);
    else if (E <= 128) TOPK(4);
    else if (E <= 256) TOPK(8);
    else TOPK(16);
#undef TOPK
}

// ---------------------------------------------------------------------------
// k_router_dec: exact logits of every token for decode-sized batches. Each logit
// is the reference's sequential f32 chain (quant/mod.rs:921-935): one rounded mul
// then one rounded add per input, ascending, bit for bit. T x (E + 1) chains run
// side by side, so the chain latency (d dependent adds) sets the time. CTA = R
// router rows (row E = the shared-expert gate) x TK tokens; lane = (row, token),
// a warp covering R rows x 32/R tokens. The CTA's whole slice (R rows and TK token
// rows, row pitch d + 4 floats so a lane's 16-byte reads of its own row fall in
// distinct banks) arrives by bulk copies issued by separate threads, in RD_NC
// chunks of the inputs with one mbarrier each, so the chains start once the first
// chunk has landed while the rest is in flight; a lane then gets
// four steps' weights and inputs from two 16-byte shared loads. The wait is
// bounded (PI_DEVERR_TIMEOUT). The last CTA to finish a token group (a ticket per
// group, taken after the logits are written and fenced) then routes the group's
// tokens (topk_token, warp per token), which saves the separate top-k launch.
// ---------------------------------------------------------------------------
constexpr int RD_NC = 4;  // chunks of the inputs, one mbarrier each
template <int R, int TK>
constexpr size_t rd_smem(int d) { return sizeof(float) * (size_t)(R + TK) * (d + 4); }
template <int R, int TK, int NPL, bool FUSE, int NTH>
__global__ __launch_bounds__(NTH) void k_router_dec(const float* __restrict__ xin, const float* __restrict__ W,
                                                       const float* __restrict__ bias, int T, int d, int E,
                                                       float* __restrict__ logits, int k, int has_shgate,
                                                       int32_t* __restrict__ idx, float* __restrict__ gates,
                                                       float* __restrict__ shscale, int32_t* __restrict__ counts,
                                                       int32_t* __restrict__ tickets, int fuse, uint32_t* err) {
    static_assert(!FUSE || NTH == TK_WARPS * 32, "one warp per top-k token slot");
    static_assert(R * TK <= NTH, "a lane per (row, token)");
    extern __shared__ __align__(16) float rd_sm[];
    __shared__ __align__(8) uint64_t full[RD_NC];
    const int tid = threadIdx.x;
    const int e0 = blockIdx.x * R, t0 = blockIdx.y * TK;
    const int nt = min(TK, T - t0), nrow = min(R, E + 1 - e0);
    const int pitch = d + 4, dc = d / RD_NC;
    if (tid == 0) {
        for (int c = 0; c < RD_NC; ++c) pitc::mbar_init(&full[c], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int c = 0; c < RD_NC; ++c) pitc::mbar_expect_tx(&full[c], (uint32_t)((nrow + nt) * dc * 4));
    }
    __syncthreads();
    // copy (row q, chunk c) by thread q + (R + TK) c: rows 0..R-1 router, R.. tokens.
    // The router rows are constant, so their copies start before the programmatic-launch
    // wait and overlap the tail of the kernel that writes the token rows.
    for (int q = tid; q < R * RD_NC; q += NTH) {
        const int row = q % R, c = q / R;
        if (row < nrow)
            pitc::bulk_load(rd_sm + row * pitch + c * dc, W + (int64_t)(e0 + row) * d + c * dc, (uint32_t)dc * 4,
                            &full[c]);
    }
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    for (int q = tid; q < TK * RD_NC; q += NTH) {
        const int row = q % TK, c = q / TK;
        if (row < nt)
            pitc::bulk_load(rd_sm + (R + row) * pitch + c * dc, xin + (int64_t)(t0 + row) * d + c * dc,
                            (uint32_t)dc * 4, &full[c]);
    }
    const int r = tid % R, tk = tid / R;
    const bool live = r < nrow && tk < nt;  // lanes tid >= R * TK have tk >= TK >= nt
    const float* wr = rd_sm + r * pitch;
    const float* xv = rd_sm + (R + tk) * pitch;
    float acc = 0.0f;
    for (int c = 0; c < RD_NC; ++c) {
        if (!pitc::mbar_wait(&full[c], 0)) {
            if (tid == 0) atomicOr(err, PI_DEVERR_TIMEOUT);
            return;
        }
        if (!live) continue;
#pragma unroll 32  // 5.0 cycles per step against 6.0 at 8 (one chain per lane, measured)
        for (int i = c * dc; i < (c + 1) * dc; i += 4) {
            const float4 w4 = *reinterpret_cast<const float4*>(wr + i);
            const float4 x4 = *reinterpret_cast<const float4*>(xv + i);
            acc = fadd(acc, fmul(w4.x, x4.x));
            acc = fadd(acc, fmul(w4.y, x4.y));
            acc = fadd(acc, fmul(w4.z, x4.z));
            acc = fadd(acc, fmul(w4.w, x4.w));
        }
    }
    if (live) {
        const int e = e0 + r;
        if (bias && e < E) acc = fadd(acc, bias[e]);
        logits[(size_t)(t0 + tk) * (E + 1) + e] = acc;
    }
    if (!FUSE || !fuse) return;
    __shared__ float s_p[TK_WARPS][32 * NPL];
    __shared__ int s_sel[TK_WARPS][32];
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&tickets[blockIdx.y], 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int warp = tid >> 5, lane = tid & 31;
    for (int j = warp; j < nt; j += TK_WARPS)
        topk_token<NPL>(logits, t0 + j, E, k, has_shgate, idx, gates, shscale, counts, s_p[warp], s_sel[warp], lane);
}



// ---------------------------------------------------------------------------
// Certified tensor-core routing for prefill batches.
//
// k_split_tokens: x [T][d] -> f16 hi/lo xh, xl (x = hi + lo + r, |r| <= 2^-22 |x|
// plus 2^-25 where lo is subnormal) and an upper bound of ||x_t||_2 (+inf when
// a value is not finite or |x| >= 2^15, which sends the token to the exact path).
// grid T, block 256.
// ---------------------------------------------------------------------------
constexpr int KC_ROUTER = 32, TC_PER_LANE = 8, TC_WARPS = 4;

__global__ __launch_bounds__(256) void k_split_tokens(const float* __restrict__ x, int d, __half* __restrict__ xh,
                                                      __half* __restrict__ xl, float* __restrict__ xnorm) {
    split_row(x + (size_t)blockIdx.x * d, blockIdx.x, d, xh, xl, xnorm);
}

// ---------------------------------------------------------------------------
// k_router_cand: a warp walks RC_TPW tokens. From the fast logits l_e (tensor cores) it
// builds intervals [l_e - eps_e, l_e + eps_e] that contain the reference's
// logit (sequential f32 sum, quant/mod.rs:921-935, then + bias), with
//   eps_e = 2 ((4d + 64) u ||x|| ||w_e|| + 2^-23 sqrt(d) (||w_e|| + 2^-rs ||x||))
//           + 2^-21 (|l_e| + |b_e|),  u = 2^-24:
// the reference's own error (<= d u sum |x_i w_i|), the tensor-core sums (at
// most 17 units of 2^-23 per k16 step relative to the magnitudes involved),
// the hi/lo representation (12 u |x_i w_i|, and 2^-25 where a part is
// subnormal), and the final f32 operations; sum |x_i w_i| <= ||x|| ||w_e||.
// Every expert whose upper end reaches the k-th largest lower end is a
// candidate (the true top-k are among them, at most 31 kept). The candidates'
// rows (and the shared-expert gate row) of consecutive tokens join a batch of
// up to 32 rows; each lane of the warp then runs the reference's exact chain for
// one row of the batch, against its own token's x, and each token's top-k is
// taken on its exact logits. The
// token is certified when the k-th exact logit clears both the next candidate
// and every non-candidate's upper end by 2^-16 (1 + |l_k - max|), so that the
// reference's choice by rounded probability (ties to the lowest index) is the
// same. Certified tokens get idx (ascending), gates from the exact logits and
// the shared gate; the others are appended to flag_list for the exact path.
// ---------------------------------------------------------------------------
constexpr int RC_TT = 64;      // tokens per CTA at most
constexpr int RC_THR = 512;    // threads per CTA
constexpr int RC_JPT = 4;      // exact chains per thread at most (64 tokens x 32 rows)
constexpr int RC_CH = 64;      // floats of each staged row per piece
constexpr int RC_NS = 2;       // pieces in flight
constexpr int RC_PITCH = RC_CH + 4;  // +4: 16-byte loads of rows 1 .. 7 apart hit distinct banks
constexpr int RC_MAXR = 257;   // staged router rows: E <= 256 experts + the shared-expert gate row
size_t router_cand_smem() { return (size_t)RC_NS * (RC_TT + RC_MAXR) * RC_PITCH * 4; }

__global__ __launch_bounds__(RC_THR, 1) void k_router_cand(
    const float* __restrict__ logits, const float* __restrict__ xnorm, const float* __restrict__ wnrm, int rs,
    const float* __restrict__ xin, const float* __restrict__ W, const float* __restrict__ bias, int T, int tt, int d,
    int E, int k, int has_shgate, int32_t* __restrict__ idx, float* __restrict__ gates, float* __restrict__ shscale,
    int32_t* __restrict__ counts, int32_t* __restrict__ flag_list, int32_t* __restrict__ n_flag) {
    extern __shared__ __align__(16) float rc_sm[];  // RC_NS pieces of {tt x rows, the used router rows}
    __shared__ uint8_t s_cand[RC_TT][32];           // candidates of each token (expert ids < 256)
    __shared__ int s_nc[RC_TT], s_joff[RC_TT + 1];  // candidates (-1: flagged), first chain of each token
    __shared__ float s_max[RC_TT];                  // largest upper end among a token's non-candidates
    __shared__ uint32_t s_used[9];                  // router rows some token of the tile needs (bit E: gate row)
    __shared__ int16_t s_rslot[RC_MAXR];            // router row -> staged slot
    __shared__ int16_t s_rows[RC_MAXR];             // staged slot -> router row
    __shared__ float s_ex[RC_TT * 32];              // exact logits, by chain
    __shared__ int s_nrows;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarp = RC_THR / 32;
    const int t0 = blockIdx.x * tt, ntok = min(tt, T - t0);
    if (ntok <= 0) return;
    const float c1 = 2.0f * (4.0f * d + 64.0f) * 0x1p-24f;
    const float cab = 2.0f * sqrtf((float)d) * 0x1p-23f;
    if (tid < 9) s_used[tid] = 0;
    __syncthreads();
    // ---- candidates, one warp per token
    for (int sl = warp; sl < ntok; sl += nwarp) {
        const int t = t0 + sl;
        const float nx = xnorm[t];
        const float* lr = logits + (size_t)t * (E + 1);
        const float sx = ldexpf(nx, -rs);
        float lo_[TC_PER_LANE], up_[TC_PER_LANE];
        bool bad = !(nx < INFINITY);
#pragma unroll
        for (int j = 0; j < TC_PER_LANE; ++j) {
            const int e = lane + 32 * j;
            lo_[j] = up_[j] = -INFINITY;
            if (e < E) {
                const float l = lr[e], b = bias ? fabsf(bias[e]) : 0.0f, wn = wnrm[e];
                const float eps = c1 * nx * wn + cab * (wn + sx) + 0x1p-21f * (fabsf(l) + b);
                lo_[j] = l - eps;
                up_[j] = l + eps;
                bad |= !(fabsf(l) < INFINITY) || !(eps < INFINITY);
            }
        }
        // tau = k-th largest lower end
        uint32_t taken = 0;
        float tau = -INFINITY;
        for (int r = 0; r < k; ++r) {
            float bl = -INFINITY;
            int bi = 0x7fffffff;
#pragma unroll
            for (int j = 0; j < TC_PER_LANE; ++j) {
                const int e = lane + 32 * j;
                if (e < E && !((taken >> j) & 1u) && (lo_[j] > bl || (lo_[j] == bl && e < bi))) { bl = lo_[j]; bi = e; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ol = __shfl_xor_sync(0xffffffffu, bl, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ol > bl || (ol == bl && oi < bi)) { bl = ol; bi = oi; }
            }
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
            tau = bl;
        }
        // candidates: upper end >= tau (at most 31 kept)
        int nc = 0;
        float maxout = -INFINITY;
#pragma unroll
        for (int j = 0; j < TC_PER_LANE; ++j) {
            const int e = lane + 32 * j;
            const bool cand = e < E && up_[j] >= tau;
            const unsigned bal = __ballot_sync(0xffffffffu, cand);
            const int pos = nc + __popc(bal & ((1u << lane) - 1u));
            if (cand && pos < 31) s_cand[sl][pos] = (uint8_t)e;
            nc += __popc(bal);
            if (e < E && !cand) maxout = fmaxf(maxout, up_[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) maxout = fmaxf(maxout, __shfl_xor_sync(0xffffffffu, maxout, o));
        bad |= nc > 31;
        if (__any_sync(0xffffffffu, bad)) {
            if (lane == 0) {
                flag_list[atomicAdd(n_flag, 1)] = t;
                s_nc[sl] = -1;
            }
            continue;
        }
        __syncwarp();
        if (lane < nc) atomicOr(&s_used[s_cand[sl][lane] >> 5], 1u << (s_cand[sl][lane] & 31));
        if (lane == 0) {
            s_nc[sl] = nc;
            s_max[sl] = maxout;
            if (has_shgate) atomicOr(&s_used[E >> 5], 1u << (E & 31));
        }
    }
    __syncthreads();
    // ---- the tile's router rows (ascending) and its chains: token sl's chains are
    // s_joff[sl] .. s_joff[sl + 1] - 1, its candidates in order, then its gate row
    if (warp == 0) {
        uint32_t wv = lane < 9 ? s_used[lane] : 0u;
        int pre = __popc(wv);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, pre, o);
            if (lane >= o) pre += v;
        }
        int base = pre - __popc(wv);
        for (; wv; wv &= wv - 1) {
            const int e = 32 * lane + __ffs(wv) - 1;
            s_rslot[e] = (int16_t)base;
            s_rows[base++] = (int16_t)e;
        }
        if (lane == 31) s_nrows = pre;
    } else if (warp == 1) {
        int run = 0;
        for (int s0 = 0; s0 < ntok; s0 += 32) {
            const int sl = s0 + lane;
            const int n = sl < ntok && s_nc[sl] >= 0 ? s_nc[sl] + (has_shgate ? 1 : 0) : 0;
            int pre = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, pre, o);
                if (lane >= o) pre += v;
            }
            if (sl < ntok) s_joff[sl] = run + pre - n;
            run += __shfl_sync(0xffffffffu, pre, 31);
        }
        if (lane == 0) s_joff[ntok] = run;
    }
    __syncthreads();
    const int nrows = s_nrows, njobs = s_joff[ntok];
    // ---- exact chains (reference order, no FMA): thread takes chains tid + RC_THR m
    int xo[RC_JPT], wo[RC_JPT];
    float acc[RC_JPT];
#pragma unroll
    for (int m = 0; m < RC_JPT; ++m) {
        acc[m] = 0.0f;
        xo[m] = wo[m] = 0;
        const int jb = tid + RC_THR * m;
        if (jb < njobs) {
            int sl = 0;  // the chain's token: last sl with s_joff[sl] <= jb
            for (int b = 32; b > 0; b >>= 1)
                if (sl + b < ntok && s_joff[sl + b] <= jb) sl += b;
            const int j = jb - s_joff[sl];
            const int row = j < s_nc[sl] ? s_cand[sl][j] : E;
            xo[m] = sl * RC_PITCH;
            wo[m] = (tt + s_rslot[row]) * RC_PITCH;
        }
    }
    const int piece = (tt + nrows) * RC_PITCH;  // floats of one staged piece
    // piece p of every staged row, 16 bytes per cp.async
    auto stage = [&](int p) {
        float* dst = rc_sm + (p % RC_NS) * piece;
        for (int q = tid; q < (ntok + nrows) * (RC_CH / 4); q += RC_THR) {
            const int r = q / (RC_CH / 4), c4 = q % (RC_CH / 4);
            const float* src = r < ntok ? xin + (size_t)(t0 + r) * d : W + (size_t)s_rows[r - ntok] * d;
            const int so = (r < ntok ? r : tt + r - ntok) * RC_PITCH + 4 * c4;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst + so)),
                         "l"(src + p * RC_CH + 4 * c4)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const int np = d / RC_CH;
    for (int p = 0; p < RC_NS - 1; ++p) {
        if (p < np) stage(p);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int p = 0; p < np; ++p) {
        asm volatile("cp.async.wait_group %0;" ::"n"(RC_NS - 2) : "memory");
        __syncthreads();  // piece p landed for every thread; piece p - 1's buffer is free
        if (p + RC_NS - 1 < np) stage(p + RC_NS - 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        const float* base = rc_sm + (p % RC_NS) * piece;
#pragma unroll
        for (int m = 0; m < RC_JPT; ++m) {
            if (tid + RC_THR * m >= njobs) break;
            const float* xr = base + xo[m];
            const float* wr = base + wo[m];
            float a = acc[m];
#pragma unroll
            for (int i = 0; i < RC_CH; i += 4) {
                const float4 wv = *reinterpret_cast<const float4*>(wr + i);
                const float4 xv = *reinterpret_cast<const float4*>(xr + i);
                a = fadd(a, fmul(wv.x, xv.x));
                a = fadd(a, fmul(wv.y, xv.y));
                a = fadd(a, fmul(wv.z, xv.z));
                a = fadd(a, fmul(wv.w, xv.w));
            }
            acc[m] = a;
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
    for (int m = 0; m < RC_JPT; ++m) {
        const int jb = tid + RC_THR * m;
        if (jb < njobs) {
            const int row = s_rows[wo[m] / RC_PITCH - tt];
            s_ex[jb] = (row < E && bias) ? fadd(acc[m], bias[row]) : acc[m];
        }
    }
    __syncthreads();
    // ---- per token: top-k on the exact logits, certification, gates
    for (int sl = warp; sl < ntok; sl += nwarp) {
        const int nc = s_nc[sl];
        if (nc < 0) continue;
        const int t = t0 + sl, off = s_joff[sl];
        const float maxout = s_max[sl];
        const float gl = has_shgate ? s_ex[off + nc] : 0.0f;  // gate row's logit
        // top-k on the exact logits (ties to the lowest index)
        const float myv = lane < nc ? s_ex[off + lane] : -INFINITY;
        const int myi = lane < nc ? (int)s_cand[sl][lane] : 0x7fffffff;
        float m = myv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bool sel = false;
        float lk = -INFINITY;
        for (int r = 0; r < k; ++r) {
            float bv = sel ? -INFINITY : myv;
            int bi = sel ? 0x7fffffff : myi;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (lane < nc && myi == bi) sel = true;
            lk = bv;
        }
        float nxt = (lane < nc && !sel) ? myv : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) nxt = fmaxf(nxt, __shfl_xor_sync(0xffffffffu, nxt, o));
        const float delta = 0x1p-16f * (1.0f + fabsf(lk - m));
        if (!(lk - nxt > delta && lk - maxout > delta)) {
            if (lane == 0) flag_list[atomicAdd(n_flag, 1)] = t;
            continue;
        }
        // ascending order of the selected experts (model/mod.rs:1303), gates from the exact logits
        const unsigned selm = __ballot_sync(0xffffffffu, sel);
        int rank = 0;
        for (unsigned b = selm; b; b &= b - 1) {
            const int ln = __ffs(b) - 1;
            rank += __shfl_sync(0xffffffffu, myi, ln) < myi;
        }
        const float p = sel ? exp_cr(fsub(myv, m)) : 0.0f;
        float ssum = 0.0f;
        for (int r = 0; r < k; ++r) {  // sequential, ascending expert order
            const unsigned b = __ballot_sync(0xffffffffu, sel && rank == r);
            ssum = fadd(ssum, __shfl_sync(0xffffffffu, p, __ffs(b) - 1));
        }
        if (sel) {
            idx[(size_t)t * k + rank] = myi;
            gates[(size_t)t * k + rank] = ssum > 0.0f ? fdiv(p, ssum) : p;
            atomicAdd(&counts[myi], 1);
        }
        if (lane == 0 && shscale) shscale[t] = has_shgate ? sigmoid_ref(gl) : 1.0f;
    }
}

// ---------------------------------------------------------------------------
// k_topk_api: MoeRouter::route of the standalone operator API
// (moe/mod.rs:69-108): top-k by logit (ties to the lowest index), ordered by
// descending logit, then ops::softmax over the k selected (ops.rs:160-180:
// max, v = exp(v - max), sequential sum, v *= 1/sum).
// ---------------------------------------------------------------------------
__global__ __launch_bounds__(TK_WARPS * 32) void k_topk_api(const float* __restrict__ logits, int T, int E, int k,
                                                            int32_t* __restrict__ idx, float* __restrict__ wts) {
    __shared__ int s_sel[TK_WARPS][32];
    __shared__ float s_v[TK_WARPS][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * TK_WARPS + warp;
    if (t >= T) return;
    const float* lr = logits + (size_t)t * (E + 1);
    float l[TK_PER_LANE];
#pragma unroll
    for (int j = 0; j < TK_PER_LANE; ++j) {
        int e = lane + 32 * j;
        l[j] = (e < E) ? lr[e] : -INFINITY;
    }
    uint32_t taken = 0;
    for (int r = 0; r < k; ++r) {
        float bp = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < TK_PER_LANE; ++j) {
            int e = lane + 32 * j;
            if (e < E && !((taken >> j) & 1u) && (l[j] > bp || (l[j] == bp && e < bi))) { bp = l[j]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float op = __shfl_xor_sync(0xffffffffu, bp, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (op > bp || (op == bp && oi < bi)) { bp = op; bi = oi; }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        if (lane == 0) { s_sel[warp][r] = bi; s_v[warp][r] = bp; }
    }
    __syncwarp();
    if (lane == 0) {
        float mx = -INFINITY;
        for (int r = 0; r < k; ++r) mx = fmaxf(mx, s_v[warp][r]);
        float sum = 0.0f;
        for (int r = 0; r < k; ++r) {
            const float v = exp_cr(fsub(s_v[warp][r], mx));
            s_v[warp][r] = v;
            sum = fadd(sum, v);
        }
        const float inv = fdiv(1.0f, sum);
        for (int r = 0; r < k; ++r) {
            idx[(size_t)t * k + r] = s_sel[warp][r];
            wts[(size_t)t * k + r] = fmul(s_v[warp][r], inv);
        }
    }
}

// ---------------------------------------------------------------------------
// k_dispatch: one CTA per expert (+ CTA E for the shared expert's items).
// offsets[e] = sum counts[<e]; perm lists the tokens routed to e ascending;
// slot_of[t*k+j] = slot of (token t, its j-th expert); work items of <= TG
// tokens: item = {expert, first slot, n tokens}. Shared-expert slots follow
// the T*k routed slots (slot T*k + t for token t).
// ---------------------------------------------------------------------------
__device__ int block_sum_int(int v, int* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    int s = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
    return s;
}

template <int DPT>  // tokens ranked per thread per round
__global__ __launch_bounds__(256) void k_dispatch(const int32_t* __restrict__ idx, const int32_t* __restrict__ counts,
                                                  int T, int k, int E, int has_shared, int32_t* __restrict__ offsets,
                                                  int32_t* __restrict__ perm, int32_t* __restrict__ slot_of,
                                                  int4* __restrict__ items, int32_t* __restrict__ n_items, int tg) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    __shared__ int red[8];
    __shared__ int s_wsum[8];
    const int e = blockIdx.x;
    int s_off = 0, s_items = 0;
    for (int i = threadIdx.x; i < e; i += blockDim.x) {
        int c = counts[i];
        s_off += c;
        s_items += (c + tg - 1) / tg;
    }
    const int off = block_sum_int(s_off, red);
    const int ibase = block_sum_int(s_items, red);
    if (e == E) {  // shared-expert items + total item count
        int n_routed_items = ibase;
        int nsh = has_shared ? (T + tg - 1) / tg : 0;
        for (int q = threadIdx.x; q < nsh; q += blockDim.x) {
            const int lo = (int)((int64_t)T * q / nsh), hi = (int)((int64_t)T * (q + 1) / nsh);
            items[n_routed_items + q] = make_int4(E, T * k + lo, hi - lo, 0);
        }
        if (threadIdx.x == 0) *n_items = n_routed_items + nsh;
        return;
    }
    const int cnt = counts[e];
    if (threadIdx.x == 0 && offsets) offsets[e] = off;
    // cnt slots in nI items of balanced sizes (each <= tg)
    const int nI = (cnt + tg - 1) / tg;
    for (int q = threadIdx.x; q < nI; q += blockDim.x) {
        const int lo = (int)((int64_t)cnt * q / nI), hi = (int)((int64_t)cnt * (q + 1) / nI);
        items[ibase + q] = make_int4(e, off + lo, hi - lo, 0);
    }
    if (cnt == 0) return;
    // slots of expert e in ascending token order: each thread checks DPT consecutive
    // tokens per round, a block scan of the per-thread match counts gives the ranks
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int base = 0;
    for (int t0 = 0; t0 < T; t0 += blockDim.x * DPT) {
        int jsel[DPT], mine = 0;
#pragma unroll
        for (int q = 0; q < DPT; ++q) {
            const int t = t0 + threadIdx.x * DPT + q;
            jsel[q] = -1;
            if (t < T)
                for (int j = 0; j < k; ++j)
                    if (idx[(size_t)t * k + j] == e) jsel[q] = j;
            mine += jsel[q] >= 0;
        }
        int incl = mine;  // inclusive warp scan of the match counts
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        __syncthreads();  // s_wsum of the previous round is consumed
        if (lane == 31) s_wsum[warp] = incl;
        __syncthreads();
        int before = 0, total = 0;
        for (int w = 0; w < nw; ++w) {
            if (w < warp) before += s_wsum[w];
            total += s_wsum[w];
        }
        int slot = off + base + before + incl - mine;
#pragma unroll
        for (int q = 0; q < DPT; ++q) {
            if (jsel[q] >= 0) {
                const int t = t0 + threadIdx.x * DPT + q;
                perm[slot] = t;
                slot_of[(size_t)t * k + jsel[q]] = slot;
                ++slot;
            }
        }
        base += total;
    }
}

// ---------------------------------------------------------------------------
// Large-batch dispatch: the same outputs as k_dispatch (offsets, the stable
// permutation, slot_of, balanced work items) from a chunked counting sort.
//   k_disp_count   per chunk of DC tokens, per-expert counts (cc[chunk][e]);
//   k_disp_scan    per expert an exclusive scan over chunks, offsets and items;
//   k_disp_scatter per chunk a bitmask [e][token] in shared memory: the rank of
//                  (token t, expert e) in the chunk is the popcount of e's bits
//                  below t, so slots stay in ascending token order.
// ---------------------------------------------------------------------------
constexpr int DC = 256;        // tokens per dispatch chunk (one per thread)
constexpr int DC_MAXE = 512;   // experts a dispatch CTA keeps in shared memory

__global__ __launch_bounds__(DC) void k_disp_count(const int32_t* __restrict__ idx, int T, int k, int E,
                                                   int32_t* __restrict__ cc) {
    __shared__ int h[DC_MAXE];
    for (int e = threadIdx.x; e < E; e += DC) h[e] = 0;
    __syncthreads();
    const int t = blockIdx.x * DC + threadIdx.x;
    if (t < T)
        for (int j = 0; j < k; ++j) {
            const int e = idx[(size_t)t * k + j];
            if ((unsigned)e < (unsigned)E) atomicAdd(&h[e], 1);
        }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += DC) cc[(size_t)blockIdx.x * E + e] = h[e];
}

// Shared-expert items cover n_sh slots starting at T*k, or (n_routed_out != NULL) right
// after the realised routed slots, whose count is then written to *n_routed_out.
__global__ __launch_bounds__(512) void k_disp_scan(int32_t* __restrict__ cc, int nchunk, int T, int k, int E,
                                                   int n_sh, int tg, int32_t* __restrict__ offsets,
                                                   int4* __restrict__ items, int32_t* __restrict__ n_items,
                                                   int32_t* __restrict__ n_routed_out) {
    __shared__ int s_w[16], s_wi[16];
    const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
    int cnt = 0;
    if (e < E)
        for (int c0 = 0; c0 < nchunk; c0 += 16) {  // 16 chunks' counts in flight per round trip
            int v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = c0 + j < nchunk ? cc[(size_t)(c0 + j) * E + e] : 0;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (c0 + j < nchunk) {
                    cc[(size_t)(c0 + j) * E + e] = cnt;
                    cnt += v[j];
                }
        }
    const int ni = (cnt + tg - 1) / tg;
    int a = cnt, b = ni;  // inclusive block scans of counts and item counts
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ya = __shfl_up_sync(0xffffffffu, a, o), yb = __shfl_up_sync(0xffffffffu, b, o);
        if (lane >= o) { a += ya; b += yb; }
    }
    if (lane == 31) { s_w[warp] = a; s_wi[warp] = b; }
    __syncthreads();
    int pa = 0, pb = 0, ta = 0, tb = 0;
    for (int w = 0; w < 16; ++w) {
        if (w < warp) { pa += s_w[w]; pb += s_wi[w]; }
        ta += s_w[w];
        tb += s_wi[w];
    }
    const int off = pa + a - cnt, ibase = pb + b - ni;
    if (e < E) {
        if (offsets) offsets[e] = off;
        for (int q = 0; q < ni; ++q) {
            const int lo = (int)((int64_t)cnt * q / ni), hi = (int)((int64_t)cnt * (q + 1) / ni);
            items[ibase + q] = make_int4(e, off + lo, hi - lo, 0);
        }
    }
    const int nsh = (n_sh + tg - 1) / tg;
    const int sbase = n_routed_out ? ta : T * k;
    for (int q = threadIdx.x; q < nsh; q += blockDim.x) {
        const int lo = (int)((int64_t)n_sh * q / nsh), hi = (int)((int64_t)n_sh * (q + 1) / nsh);
        items[tb + q] = make_int4(E, sbase + lo, hi - lo, 0);
    }
    if (threadIdx.x == 0) {
        *n_items = tb + nsh;
        if (n_routed_out) *n_routed_out = ta;
    }
}

__global__ __launch_bounds__(DC) void k_disp_scatter(const int32_t* __restrict__ idx, int T, int k, int E,
                                                     const int32_t* __restrict__ cc,
                                                     const int32_t* __restrict__ offsets, int32_t* __restrict__ perm,
                                                     int32_t* __restrict__ slot_of) {
    __shared__ uint32_t mask[DC_MAXE * (DC / 32)];
    for (int i = threadIdx.x; i < E * (DC / 32); i += DC) mask[i] = 0;
    __syncthreads();
    const int t = blockIdx.x * DC + threadIdx.x, w = threadIdx.x >> 5;
    const uint32_t bit = 1u << (threadIdx.x & 31);
    if (t < T)
        for (int j = 0; j < k; ++j) {
            const int e = idx[(size_t)t * k + j];
            if ((unsigned)e < (unsigned)E) atomicOr(&mask[e * (DC / 32) + w], bit);
        }
    __syncthreads();
    if (t >= T) return;
    for (int j = 0; j < k; ++j) {
        const int e = idx[(size_t)t * k + j];
        if ((unsigned)e >= (unsigned)E) continue;
        const uint32_t* me = &mask[e * (DC / 32)];
        int r = __popc(me[w] & (bit - 1));
        for (int x = 0; x < w; ++x) r += __popc(me[x]);
        const int slot = offsets[e] + cc[(size_t)blockIdx.x * E + e] + r;
        perm[slot] = t;
        slot_of[(size_t)t * k + j] = slot;
    }
}

// ---------------------------------------------------------------------------
// Expert GEMV kernels.
// ---------------------------------------------------------------------------
PI_DEV int slot_token(const ExpertArgs& a, bool sh, int slot) { return sh ? slot - a.n_routed : a.perm[slot]; }

// Q8_0 gate+up: CTA = 2 * GU_WARPS rows of one expert (2 rows per warp, gate
// and up = 4 row-vectors per warp), CPL = d/512 16-byte chunks per lane per row
// (lane l holds chunks l + 32c; chunks 2m, 2m+1 form 32-element block m).
// Small CTAs (64 threads, ~17 KB of shared memory, eight per SM) retire and are
// replaced one by one, so an SM's weight loads overlap other CTAs' arithmetic
// without waiting for a large CTA's slowest warp (C2 T=64: 106 us with 256-thread
// CTAs, 100.5 with 128, 99.9 with 64).
//
// The sums keep the reference's order exactly (matvec_q8_0_sse_range,
// quant/mod.rs:835-871): per block an exact int32 dot, the term
// (float)sumi * (d_w * d_x), and the terms added sequentially in block order.
// Terms are staged in shared memory; lane (rv, token) of each warp then runs
// the sequential chain for one (row-vector, token) pair. h is therefore the
// reference's h bit for bit (up to its expf rounding), so the Q8_0
// re-quantisation of h in k_down_q8 makes the same integer choices.
constexpr int GU_TB = 8;    // tokens per batch: 4 row-vectors x 8 tokens = 32 chains per warp
constexpr int GU_WARPS = 2;            // warps per CTA (2 rows each)
constexpr int GU_ROWS = 2 * GU_WARPS;  // rows per CTA
template <int CPL>
__global__ __launch_bounds__(GU_WARPS * 32, 16 / GU_WARPS) void k_gateup_q8(ExpertArgs a) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    constexpr int NB = 16 * CPL;   // blocks per row
    constexpr int STRIDE = NB + 4; // padded chain stride (floats): conflict-free 16-byte reads
    extern __shared__ __align__(16) float smem[];
    float* terms = smem + (threadIdx.x >> 5) * (4 * GU_TB * STRIDE);
    __shared__ float res[GU_WARPS][4][GU_TB];
    const int it = blockIdx.y;
    if (it >= *a.n_items) return;
    const int4 item = a.items[it];
    const bool sh = (item.x == a.E);
    const int d = a.d, f = a.f, nb = d / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rA = blockIdx.x * GU_ROWS + 2 * warp;
    const size_t mat = sh ? 0 : (size_t)item.x * f;
    const int8_t* G = (const int8_t*)(sh ? a.gs : a.g) + (mat + rA) * d;
    const int8_t* U = (const int8_t*)(sh ? a.us : a.u) + (mat + rA) * d;
    const __half* GD = (sh ? a.gsd : a.gd) + (mat + rA) * nb;
    const __half* UD = (sh ? a.usd : a.ud) + (mat + rA) * nb;
    // rows are lane-tiled (pi_tile_gateup_mats): the lane's c-th 16-byte load is
    // half (c % 2) of block lane + 32 * (c / 2), and each load is a contiguous
    // 512-byte segment of the row for the warp.
    constexpr int BPL = CPL / 2;  // whole blocks per lane
    int4 w[4][CPL];
    float sw[4][BPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        const int off = (c * 32 + lane) * 16;
        w[0][c] = ld_stream(G + off);
        w[1][c] = ld_stream(U + off);
        w[2][c] = ld_stream(G + d + off);
        w[3][c] = ld_stream(U + d + off);
    }
#pragma unroll
    for (int bb = 0; bb < BPL; ++bb) {
        const int b = lane + 32 * bb;
        sw[0][bb] = __half2float(GD[b]);
        sw[1][bb] = __half2float(UD[b]);
        sw[2][bb] = __half2float(GD[nb + b]);
        sw[3][bb] = __half2float(UD[nb + b]);
    }
    const int crv = lane >> 3, ctk = lane & 7;  // this lane's chain
    for (int t0 = 0; t0 < item.z; t0 += GU_TB) {
        const int nt = min(GU_TB, item.z - t0);
        for (int tk = 0; tk < nt; ++tk) {
            const int slot = item.y + t0 + tk;
            const int tok = slot_token(a, sh, slot);
            const int8_t* xr = a.xq + (size_t)tok * d;
            const float* sr = a.xs + (size_t)tok * nb;
#pragma unroll
            for (int bb = 0; bb < BPL; ++bb) {
                const int b = lane + 32 * bb;
                const int4 x0 = *reinterpret_cast<const int4*>(xr + b * 32);
                const int4 x1 = *reinterpret_cast<const int4*>(xr + b * 32 + 16);
                const float sx = sr[b];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int4 w0 = w[r][2 * bb], w1 = w[r][2 * bb + 1];
                    int s = dp4a(w0.x, x0.x, 0);
                    s = dp4a(w0.y, x0.y, s);
                    s = dp4a(w0.z, x0.z, s);
                    s = dp4a(w0.w, x0.w, s);
                    s = dp4a(w1.x, x1.x, s);
                    s = dp4a(w1.y, x1.y, s);
                    s = dp4a(w1.z, x1.z, s);
                    s = dp4a(w1.w, x1.w, s);
                    terms[(r * GU_TB + tk) * STRIDE + b] = fmul((float)s, fmul(sw[r][bb], sx));
                }
            }
        }
        __syncwarp();
        if (ctk < nt) {
            const float4* tp = reinterpret_cast<const float4*>(terms + (crv * GU_TB + ctk) * STRIDE);
            float acc = 0.0f;
#pragma unroll
            for (int q = 0; q < NB / 4; ++q) {
                const float4 v = tp[q];
                acc = fadd(acc, v.x);
                acc = fadd(acc, v.y);
                acc = fadd(acc, v.z);
                acc = fadd(acc, v.w);
            }
            res[warp][crv][ctk] = acc;
        }
        __syncwarp();
        if (lane < 2 * GU_TB) {
            const int r = lane / GU_TB, tk = lane % GU_TB;  // row rA + r
            if (tk < nt)
                a.hf[(size_t)(item.y + t0 + tk) * f + rA + r] = swiglu_ref(res[warp][2 * r][tk], res[warp][2 * r + 1][tk]);
        }
        __syncwarp();
    }
}

template <int CPL>
constexpr size_t gateup_q8_smem() {
    return (size_t)GU_WARPS * 4 * GU_TB * (16 * CPL + 4) * sizeof(float);
}

// Q8_0 h re-quantisation (quant/mod.rs:698-736, as the reference's down
// matvec quantises its input): warp per 32-block of hf[slot][.].
__global__ void k_quant_h(const float* __restrict__ hf, int64_t nblk, int8_t* __restrict__ hq,
                          float* __restrict__ hs) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    // thread = four consecutive values, eight lanes per 32-block (quad_quant_q8); threads
    // past the end still take part in the shuffles of their warp
    const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const bool live = g < nblk * 8;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) v = *reinterpret_cast<const float4*>(hf + 4 * g);
    const float e[4] = {v.x, v.y, v.z, v.w};
    float sc;
    const uint32_t q = quad_quant_q8(e, &sc);
    if (!live) return;
    *reinterpret_cast<uint32_t*>(hq + 4 * g) = q;
    if ((g & 7) == 0) hs[g >> 3] = sc;
}

// Q8_0 down, streamed: a persistent CTA per SM walks work units u = (item, block of
// DS_ROWS output rows), u = blockIdx.x, blockIdx.x + gridDim.x, ... A producer
// thread bulk-copies each unit's inputs into a ring of DS_NS shared-memory stages
// (the 64 rows are one contiguous 8-row-group run of the lane-tiled layout, their
// f16 block scales, and the item's quantised h rows and scales) onto the stage's
// mbarrier, so HBM streams continuously while 8 consumer warps compute; a warp
// releases the stage on a second mbarrier. Warp w owns rows 8w .. 8w+7 of the unit,
// 4 lanes per row as in k_down_q8; block terms go to shared memory and lane c sums
// chain c = (row, token) over the row's blocks in ascending order (quant/mod.rs:
// 877-899), bit for bit. Every wait is bounded (PI_DEVERR_TIMEOUT).
constexpr int DS_ROWS = 64, DS_NS = 4, DS_THREADS = 9 * 32;
template <int CPQ>
struct DSL {
    static constexpr int F = CPQ * 64, FB = F / 32, BPQ = CPQ / 2, TS = FB + 1;
    static constexpr int W = DS_ROWS * F, S = DS_ROWS * FB * 2, H = TG * F, HS = TG * FB * 4;
    static constexpr int STAGE = W + S + H + HS;
    static constexpr size_t SMEM = (size_t)DS_NS * STAGE + sizeof(float) * 8 * 32 * TS;
};
template <int CPQ>
__global__ __launch_bounds__(DS_THREADS, 1) void k_down_q8s(ExpertArgs a, uint32_t* err) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    using L = DSL<CPQ>;
    constexpr int F = L::F, FB = L::FB, BPQ = L::BPQ, TS = L::TS;
    extern __shared__ __align__(128) uint8_t ds_sm[];
    __shared__ __align__(8) uint64_t full[DS_NS], empty[DS_NS];
    __shared__ int4 meta[DS_NS];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int d = a.d, nrb = d / DS_ROWS;
    const int n_units = *a.n_items * nrb;
    if (tid == 0) {
        for (int s = 0; s < DS_NS; ++s) {
            pitc::mbar_init(&full[s], 1);
            pitc::mbar_init(&empty[s], 8);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    bool ok = true;
    if (warp == 8) {
        if (lane == 0) {
            int k = 0;
            for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++k) {
                const int s = k % DS_NS;
                if (k >= DS_NS && !pitc::mbar_wait(&empty[s], ((k / DS_NS) - 1) & 1)) { ok = false; break; }
                const int4 item = a.items[u / nrb];
                const int rb = u % nrb;
                meta[s] = make_int4(item.x, item.y, item.z, rb);
                const bool sh = item.x == a.E;
                const size_t row0 = (sh ? 0 : (size_t)item.x * d) + (size_t)rb * DS_ROWS;
                uint8_t* st = ds_sm + (size_t)s * L::STAGE;
                pitc::mbar_expect_tx(&full[s], (uint32_t)(L::W + L::S + item.z * (F + FB * 4)));
                pitc::bulk_load(st, (const int8_t*)(sh ? a.dns : a.dn) + row0 * F, L::W, &full[s]);
                pitc::bulk_load(st + L::W, (sh ? a.dsd : a.dd) + row0 * FB, L::S, &full[s]);
                pitc::bulk_load(st + L::W + L::S, a.hq + (size_t)item.y * F, (uint32_t)(item.z * F), &full[s]);
                pitc::bulk_load(st + L::W + L::S + L::H, a.hs + (size_t)item.y * FB, (uint32_t)(item.z * FB * 4),
                                &full[s]);
            }
        }
    } else {
        float* terms = reinterpret_cast<float*>(ds_sm + (size_t)DS_NS * L::STAGE) + warp * 32 * TS;
        const int q = lane & 3, r8 = lane >> 2;
        int k = 0;
        for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++k) {
            const int s = k % DS_NS;
            if (!pitc::mbar_wait(&full[s], (k / DS_NS) & 1)) { ok = false; break; }
            const int4 m = meta[s];
            const uint8_t* st = ds_sm + (size_t)s * L::STAGE;
            // quarter q walks its blocks rotated by q (block (b + q) % BPQ at step b): the four
            // quarters of a row then read h chunks in distinct banks; only shared-memory
            // addresses rotate, registers stay statically indexed
            int4 w[CPQ];
            float sw[BPQ];
#pragma unroll
            for (int c = 0; c < CPQ; ++c)
                w[c] = *reinterpret_cast<const int4*>(st + warp * 8 * F + (((c + 2 * q) % CPQ) * 32 + lane) * 16);
            const __half* sc = reinterpret_cast<const __half*>(st + L::W) + (warp * 8 + r8) * FB + q * BPQ;
#pragma unroll
            for (int b = 0; b < BPQ; ++b) sw[b] = __half2float(sc[(b + q) % BPQ]);
            const int8_t* hq = reinterpret_cast<const int8_t*>(st + L::W + L::S);
            const float* hs = reinterpret_cast<const float*>(st + L::W + L::S + L::H);
            constexpr int DTB = 4;  // tokens per batch: 8 rows x 4 tokens = 32 chains
            for (int t0 = 0; t0 < m.z; t0 += DTB) {
                const int nt = min(DTB, m.z - t0);
                for (int j = 0; j < nt; ++j) {
                    const int8_t* hr = hq + (t0 + j) * F + q * CPQ * 16;
                    const float* hsr = hs + (t0 + j) * FB + q * BPQ;
                    float* tr = terms + (r8 * DTB + j) * TS + q * BPQ;
#pragma unroll
                    for (int b = 0; b < BPQ; ++b) {
                        const int br = (b + q) % BPQ;
                        int sum = 0;
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int4 wv = w[2 * b + h], xv = *reinterpret_cast<const int4*>(hr + (2 * br + h) * 16);
                            sum = dp4a(wv.x, xv.x, sum);
                            sum = dp4a(wv.y, xv.y, sum);
                            sum = dp4a(wv.z, xv.z, sum);
                            sum = dp4a(wv.w, xv.w, sum);
                        }
                        tr[br] = fmul((float)sum, fmul(sw[b], hsr[br]));
                    }
                }
                __syncwarp();
                const int j = lane % DTB, rr = lane / DTB;
                if (j < nt) {
                    const float* tp = terms + lane * TS;
                    float acc = 0.0f;
#pragma unroll
                    for (int b = 0; b < FB; ++b) acc = fadd(acc, tp[b]);
                    a.y[(size_t)(m.y + t0 + j) * d + m.w * DS_ROWS + warp * 8 + rr] = acc;
                }
                __syncwarp();
            }
            if (lane == 0) pitc::mbar_arrive(&empty[s]);
        }
    }
    if (!ok) atomicOr(err, PI_DEVERR_TIMEOUT);
}

// Q8_0 down: CTA = DN_ROWS output rows (8 warps x 8*DN_NP rows), 4 lanes per
// row, CPQ = f/64 chunks per lane, 8 rows per warp pass; the quantised h
// of each slot comes from k_quant_h. Each output is the reference's sequential
// sum of block terms (float)sumi * (d_w * d_h) in ascending block order
// (quant/mod.rs:877-899), bit for bit.
constexpr int DN_NP = 2;             // passes of 8 rows per warp
constexpr int DN_ROWS = 64 * DN_NP;   // rows per CTA
// term buffer of k_down_q8<CPQ>: 8 warps x 32 chains x (2 CPQ + 4) floats
constexpr size_t dn_smem(int cpq) { return sizeof(float) * 8 * 32 * (2 * cpq + 4); }
template <int CPQ>
__global__ __launch_bounds__(256, 2) void k_down_q8(ExpertArgs a) {
    constexpr int F = CPQ * 64;  // expert width
    const int it = blockIdx.y;
    if (it >= *a.n_items) return;
    const int4 item = a.items[it];
    const bool sh = (item.x == a.E);
    const int d = a.d, fb = F / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = lane & 3;
    const int rbase = blockIdx.x * DN_ROWS + warp * 8 * DN_NP + (lane >> 2);
    static_assert(DN_NP * 8 <= 32, "a warp's rows x one token fit its 32 chains");
    const size_t mat = sh ? 0 : (size_t)item.x * d;
    const int8_t* D = (const int8_t*)(sh ? a.dns : a.dn) + mat * F;
    const __half* DD = (sh ? a.dsd : a.dd) + mat * fb;
    constexpr int BPQ = CPQ / 2;  // blocks per lane
    int4 w[DN_NP][CPQ];
    float sw[DN_NP][BPQ];
#pragma unroll
    for (int p = 0; p < DN_NP; ++p) {
        const int row = rbase + 8 * p;
#pragma unroll
        for (int c = 0; c < CPQ; ++c) w[p][c] = ld_stream(D + (size_t)(row >> 3) * 8 * F + (c * 32 + lane) * 16);
#pragma unroll
        for (int b = 0; b < BPQ; ++b) sw[p][b] = __half2float(DD[(size_t)row * fb + q * BPQ + b]);
    }
    // stage the item's quantised hidden vectors (the loads overlap the weight loads above)
    __shared__ __align__(16) int8_t s_hq[TG][F];
    __shared__ float s_hs[TG][F / 32];
    for (int m = threadIdx.x; m < item.z * (F / 16); m += blockDim.x) {
        const int tk = m / (F / 16), c = m % (F / 16);
        *reinterpret_cast<int4*>(&s_hq[tk][16 * c]) =
            *reinterpret_cast<const int4*>(a.hq + (size_t)(item.y + tk) * F + 16 * c);
    }
    for (int m = threadIdx.x; m < item.z * fb; m += blockDim.x)
        s_hs[m / fb][m % fb] = a.hs[(size_t)(item.y + m / fb) * fb + m % fb];
    __syncthreads();
    // block terms go to shared memory; lane c then sums chain c = (row, token) over the
    // row's FB terms in ascending block order (quant/mod.rs:877-899)
    constexpr int FB = 4 * BPQ, TS = FB + 4;  // blocks per row, padded term stride
    constexpr int DTB = 32 / (8 * DN_NP);      // tokens per batch: 32 chains per warp
    extern __shared__ __align__(16) float dn_terms[];
    float* terms = dn_terms + warp * 32 * TS;
    const int r8 = lane >> 2;
    for (int t0 = 0; t0 < item.z; t0 += DTB) {
        const int nt = min(DTB, item.z - t0);
        for (int j = 0; j < nt; ++j) {
            const int8_t* hr = &s_hq[t0 + j][q * CPQ * 16];
            const float* hsr = &s_hs[t0 + j][q * BPQ];
            int4 hv[CPQ];
            float hsv[BPQ];
#pragma unroll
            for (int c = 0; c < CPQ; ++c) hv[c] = *reinterpret_cast<const int4*>(hr + c * 16);
#pragma unroll
            for (int b = 0; b < BPQ; ++b) hsv[b] = hsr[b];
#pragma unroll
            for (int p = 0; p < DN_NP; ++p) {
                float* tr = terms + ((p * 8 + r8) * DTB + j) * TS + q * BPQ;
#pragma unroll
                for (int b = 0; b < BPQ; ++b) {
                    int sum = 0;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int4 wv = w[p][2 * b + h], xv = hv[2 * b + h];
                        sum = dp4a(wv.x, xv.x, sum);
                        sum = dp4a(wv.y, xv.y, sum);
                        sum = dp4a(wv.z, xv.z, sum);
                        sum = dp4a(wv.w, xv.w, sum);
                    }
                    tr[b] = fmul((float)sum, fmul(sw[p][b], hsv[b]));
                }
            }
        }
        __syncwarp();
        const int j = lane % DTB, pr = lane / DTB;  // chain: token t0 + j, row pass pr / 8, row pr % 8
        if (j < nt) {
            const float* tp = terms + lane * TS;
            float acc = 0.0f;
#pragma unroll
            for (int b = 0; b < FB; ++b) acc = fadd(acc, tp[b]);
            const int row = blockIdx.x * DN_ROWS + warp * 8 * DN_NP + (pr % 8) + 8 * (pr / 8);
            a.y[(size_t)(item.y + t0 + j) * d + row] = acc;
        }
        __syncwarp();
    }
}

// Q4_0 helpers: the 16 nibble bytes of a block hold elements 2i (low) and
// 2i+1 (high) of byte i; value = (nibble - 8) * d.
PI_DEV float nib_f(uint32_t v) { return __int_as_float(0x4B000000u | v) - 8388616.0f; }  // v - 8, exact

// dot of one Q4_0 block (16 nibble bytes) with 32 f32 values held in registers
PI_DEV float q4_dot_regs(const int4 wv, const float (&xv)[32]) {
    const uint32_t wd[4] = {(uint32_t)wv.x, (uint32_t)wv.y, (uint32_t)wv.z, (uint32_t)wv.w};
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 8; ++j) s = fmaf(nib_f((wd[i] >> (4 * j)) & 15u), xv[8 * i + j], s);
    }
    return s;
}

PI_DEV void load32(const float* __restrict__ x, float (&xv)[32]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(x + 4 * i);
        xv[4 * i] = v.x;
        xv[4 * i + 1] = v.y;
        xv[4 * i + 2] = v.z;
        xv[4 * i + 3] = v.w;
    }
}

// Q4_0 gate+up with f32 activations (the reference dequantises Q4_0 and
// runs an f32 dot, quant/mod.rs:958-969). CPL = d/1024 blocks per lane per row.
template <int CPL>
__global__ __launch_bounds__(512) void k_gateup_q4(ExpertArgs a) {
    const int it = blockIdx.y;
    if (it >= *a.n_items) return;
    const int4 item = a.items[it];
    const bool sh = (item.x == a.E);
    const int d = a.d, f = a.f, nb = d / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t mat = sh ? 0 : (size_t)item.x * f;
    // one row (gate and up) at a time keeps the weights of 2 x CPL blocks in registers
#pragma unroll 1
    for (int rr = 0; rr < 2; ++rr) {
        const int row = blockIdx.x * 32 + 2 * warp + rr;
        const uint8_t* G = (const uint8_t*)(sh ? a.gs : a.g) + (mat + row) * (d / 2);
        const uint8_t* U = (const uint8_t*)(sh ? a.us : a.u) + (mat + row) * (d / 2);
        const __half* GD = (sh ? a.gsd : a.gd) + (mat + row) * nb;
        const __half* UD = (sh ? a.usd : a.ud) + (mat + row) * nb;
        int4 wg[CPL], wu[CPL];
        float sg[CPL], su[CPL];
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            const int b = lane + 32 * c;
            wg[c] = ld_stream(G + b * 16);
            wu[c] = ld_stream(U + b * 16);
            sg[c] = __half2float(GD[b]);
            su[c] = __half2float(UD[b]);
        }
#pragma unroll 1
        for (int tk = 0; tk < item.z; ++tk) {
            const int slot = item.y + tk;
            const int tok = slot_token(a, sh, slot);
            const float* xr = a.xf + (size_t)tok * d;
            float ag = 0.f, au = 0.f;
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                float xv[32];
                load32(xr + (lane + 32 * c) * 32, xv);
                ag += sg[c] * q4_dot_regs(wg[c], xv);
                au += su[c] * q4_dot_regs(wu[c], xv);
            }
            ag = warp_sum(ag);
            au = warp_sum(au);
            if (lane == 0) a.hf[(size_t)slot * f + row] = swiglu_ref(ag, au);
        }
    }
}

// Q4_0 down with f32 hidden: 4 lanes per row, BPQ = f/128 blocks per lane.
template <int BPQ>
__global__ __launch_bounds__(256) void k_down_q4(ExpertArgs a) {
    const int it = blockIdx.y;
    if (it >= *a.n_items) return;
    const int4 item = a.items[it];
    const bool sh = (item.x == a.E);
    const int d = a.d, f = a.f, fb = f / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = lane & 3;
    const size_t mat = sh ? 0 : (size_t)item.x * d;
    const uint8_t* D = (const uint8_t*)(sh ? a.dns : a.dn) + mat * (f / 2);
    const __half* DD = (sh ? a.dsd : a.dd) + mat * fb;
#pragma unroll 1
    for (int p = 0; p < 2; ++p) {
        const int row = blockIdx.x * 128 + warp * 16 + (lane >> 2) + 8 * p;
        int4 w[BPQ];
        float sw[BPQ];
#pragma unroll
        for (int b = 0; b < BPQ; ++b) {
            w[b] = ld_stream(D + (size_t)(row >> 3) * 8 * (f / 2) + (b * 32 + lane) * 16);
            sw[b] = __half2float(DD[(size_t)row * fb + q * BPQ + b]);
        }
#pragma unroll 1
        for (int tk = 0; tk < item.z; ++tk) {
            const int slot = item.y + tk;
            const float* hr = a.hf + (size_t)slot * f + q * BPQ * 32;
            float acc = 0.f;
#pragma unroll
            for (int b = 0; b < BPQ; ++b) {
                float xv[32];
                load32(hr + b * 32, xv);
                acc += sw[b] * q4_dot_regs(w[b], xv);
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (q == 0) a.y[(size_t)slot * d + row] = acc;
        }
    }
}

// ---------------------------------------------------------------------------
// k_combine: out[t] = (x[t] +) sum_j gates[t][j] * y[slot(t,j)] + s_t * y_sh[t],
// experts ascending, each step o = o + g * y (no FMA), as model/mod.rs:1525-1534.
// ---------------------------------------------------------------------------
// y_sh: the shared expert's rows [T][d], or null for rows T*k .. T*k+T-1 of y.
__global__ __launch_bounds__(256) void k_combine(const float* __restrict__ x, const float* __restrict__ y,
                                                 const float* __restrict__ gates, const int32_t* __restrict__ slot_of,
                                                 const float* __restrict__ shscale, const float* __restrict__ y_sh,
                                                 int T, int k, int d, int has_shared, int residual,
                                                 float* __restrict__ out) {
    pdl_wait();  // programmatic launch: the previous kernel of the stream is complete
    pdl_trigger();
    // thread = 4 consecutive columns (16-byte loads); each column's sum keeps the
    // reference order: routed experts ascending, then the shared expert, then x
    const int t = blockIdx.x;
    const int c = 4 * (blockIdx.y * blockDim.x + threadIdx.x);
    if (c >= d) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    // the shared row's load goes out first; for k <= 8 every slot index, gate and row is
    // requested before the sum, so the latencies overlap instead of chaining
    float4 vsh = make_float4(0.f, 0.f, 0.f, 0.f);
    if (has_shared)
        vsh = *reinterpret_cast<const float4*>(y_sh ? y_sh + (size_t)t * d + c : y + ((size_t)T * k + t) * d + c);
    if (k <= 8) {
        int sl[8];
        float gj[8];
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j < k) {
                sl[j] = slot_of[(size_t)t * k + j];
                gj[j] = gates[(size_t)t * k + j];
            }
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j < k) v[j] = *reinterpret_cast<const float4*>(y + (size_t)sl[j] * d + c);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j < k) {
                acc.x = fadd(acc.x, fmul(gj[j], v[j].x));
                acc.y = fadd(acc.y, fmul(gj[j], v[j].y));
                acc.z = fadd(acc.z, fmul(gj[j], v[j].z));
                acc.w = fadd(acc.w, fmul(gj[j], v[j].w));
            }
    } else {
        for (int j = 0; j < k; ++j) {
            const int slot = slot_of[(size_t)t * k + j];
            const float g = gates[(size_t)t * k + j];
            const float4 v = *reinterpret_cast<const float4*>(y + (size_t)slot * d + c);
            acc.x = fadd(acc.x, fmul(g, v.x));
            acc.y = fadd(acc.y, fmul(g, v.y));
            acc.z = fadd(acc.z, fmul(g, v.z));
            acc.w = fadd(acc.w, fmul(g, v.w));
        }
    }
    if (has_shared) {
        const float g = shscale[t];
        const float4 v = vsh;
        acc.x = fadd(acc.x, fmul(g, v.x));
        acc.y = fadd(acc.y, fmul(g, v.y));
        acc.z = fadd(acc.z, fmul(g, v.z));
        acc.w = fadd(acc.w, fmul(g, v.w));
    }
    if (residual) {
        const float4 xv = *reinterpret_cast<const float4*>(x + (size_t)t * d + c);
        acc.x = fadd(xv.x, acc.x);
        acc.y = fadd(xv.y, acc.y);
        acc.z = fadd(xv.z, acc.z);
        acc.w = fadd(xv.w, acc.w);
    }
    *reinterpret_cast<float4*>(out + (size_t)t * d + c) = acc;
}

// ---------------------------------------------------------------------------
// Expert parallelism (no reference counterpart: the reference runs one process).
// Rank r holds experts [r P, (r + 1) P), P = E / world. Each home (token, j) slot
// is sent to its expert's rank as one Q8_0 row (the token's quantised
// activations, as every rank would quantise them) with the expert's local id.
// ---------------------------------------------------------------------------
// Layout in three passes over chunks of EPC slots: per-(chunk, rank) counts,
// an exclusive scan in (rank, chunk) order (also the per-rank totals), then a
// stable scatter: rank r's slots are contiguous after those of ranks < r, in
// slot order.
constexpr int EPC = 1024;
__global__ __launch_bounds__(EPC) void k_ep_chunk_count(const int32_t* __restrict__ idx, int n, int per_rank,
                                                        int world, int32_t* __restrict__ cc) {
    __shared__ int c[64];
    for (int i = threadIdx.x; i < world; i += blockDim.x) c[i] = 0;
    __syncthreads();
    const int s = blockIdx.x * EPC + threadIdx.x;
    if (s < n) atomicAdd(&c[idx[s] / per_rank], 1);
    __syncthreads();
    for (int i = threadIdx.x; i < world; i += blockDim.x) cc[(size_t)blockIdx.x * world + i] = c[i];
}

// cc [nchunk][world] counts -> exclusive offsets in (rank, chunk) order; counts[r] totals. One thread.
__global__ void k_ep_scan(int32_t* __restrict__ cc, int nchunk, int world, int32_t* __restrict__ counts) {
    int run = 0;
    for (int r = 0; r < world; ++r) {
        const int start = run;
        for (int ch = 0; ch < nchunk; ++ch) {
            const int v = cc[(size_t)ch * world + r];
            cc[(size_t)ch * world + r] = run;
            run += v;
        }
        counts[r] = run - start;
    }
}

__global__ __launch_bounds__(EPC) void k_ep_scatter(const int32_t* __restrict__ idx, int n, int k, int per_rank,
                                                    int world, const int32_t* __restrict__ cc,
                                                    int32_t* __restrict__ send_tok, int32_t* __restrict__ send_eid,
                                                    int32_t* __restrict__ slot_row) {
    __shared__ int s_w[64][EPC / 32];  // per rank, per warp counts
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = EPC / 32;
    const int s = blockIdx.x * EPC + threadIdx.x;
    const int r = s < n ? idx[s] / per_rank : -1;
    for (int i = threadIdx.x; i < world * nw; i += blockDim.x) s_w[i / nw][i % nw] = 0;
    __syncthreads();
    // rank of this slot among the chunk's slots of the same destination (warp-aggregated)
    const unsigned same = __match_any_sync(0xffffffffu, r);
    const int in_warp = __popc(same & ((1u << lane) - 1u));
    if (r >= 0 && in_warp == 0) s_w[r][warp] = __popc(same);
    __syncthreads();
    if (r >= 0) {
        int before = 0;
        for (int w = 0; w < warp; ++w) before += s_w[r][w];
        const int pos = cc[(size_t)blockIdx.x * world + r] + before + in_warp;
        send_tok[pos] = s / k;
        send_eid[pos] = idx[s] - r * per_rank;
        slot_row[s] = pos;
    }
}

// send rows: send_xq[p] = xq[send_tok[p]] (d bytes), send_xs[p] = xs[send_tok[p]] (d/32 floats)
__global__ void k_ep_gather(const int8_t* __restrict__ xq, const float* __restrict__ xs,
                            const int32_t* __restrict__ send_tok, int64_t n_rows, int d, int8_t* __restrict__ send_xq,
                            float* __restrict__ send_xs) {
    const int64_t p = blockIdx.x;
    if (p >= n_rows) return;
    const int64_t t = send_tok[p];
    for (int c = threadIdx.x; c < d / 16; c += blockDim.x)
        reinterpret_cast<int4*>(send_xq + p * d)[c] = reinterpret_cast<const int4*>(xq + t * d)[c];
    for (int c = threadIdx.x; c < d / 32; c += blockDim.x) send_xs[p * (d / 32) + c] = xs[t * (d / 32) + c];
}

// expert-id histogram of the given rows
__global__ void k_ep_hist(const int32_t* __restrict__ eid, int64_t n, int32_t* __restrict__ counts) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) atomicAdd(&counts[eid[i]], 1);
}

// y_rows[r] = y[slot of row r] (routed rows: slot_of[r]; shared-expert rows: n + r)
__global__ void k_rows_from_slots(const float* __restrict__ y, const int32_t* __restrict__ slot_of, int64_t n, int d,
                                  int shared, float* __restrict__ out) {
    const int64_t r = blockIdx.x;
    if (r >= n) return;
    const int64_t s = shared ? n + r : slot_of[r];
    for (int c = threadIdx.x; c < d / 4; c += blockDim.x)
        reinterpret_cast<float4*>(out + r * d)[c] = reinterpret_cast<const float4*>(y + s * d)[c];
}

// ---------------------------------------------------------------------------
// Repack: GGUF array-of-blocks -> structure-of-arrays (one thread per block).
// ---------------------------------------------------------------------------
__global__ void k_repack_q8(const uint8_t* __restrict__ src, int64_t nblk, int8_t* __restrict__ q,
                            __half* __restrict__ dd) {
    int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const uint8_t* p = src + b * 34;
    dd[b] = __ushort_as_half((uint16_t)(p[0] | (p[1] << 8)));
    uint32_t wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        wv[i] = (uint32_t)p[2 + 4 * i] | ((uint32_t)p[3 + 4 * i] << 8) | ((uint32_t)p[4 + 4 * i] << 16) |
                ((uint32_t)p[5 + 4 * i] << 24);
    int4* o = reinterpret_cast<int4*>(q + b * 32);
    o[0] = make_int4(wv[0], wv[1], wv[2], wv[3]);
    o[1] = make_int4(wv[4], wv[5], wv[6], wv[7]);
}

__global__ void k_repack_q4(const uint8_t* __restrict__ src, int64_t nblk, uint8_t* __restrict__ q,
                            __half* __restrict__ dd) {
    int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const uint8_t* p = src + b * 18;
    dd[b] = __ushort_as_half((uint16_t)(p[0] | (p[1] << 8)));
    uint32_t wv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        wv[i] = (uint32_t)p[2 + 4 * i] | ((uint32_t)p[3 + 4 * i] << 8) | ((uint32_t)p[4 + 4 * i] << 16) |
                ((uint32_t)p[5 + 4 * i] << 24);
    *reinterpret_cast<int4*>(q + b * 16) = make_int4(wv[0], wv[1], wv[2], wv[3]);
}

// Lane-tiled layout for the down projections. The down kernels read a row
// with 4 lanes (quarter q of row r) and 8 rows per warp; storing each group of
// 8 rows as [chunk c][lane = 4*(r%8) + q][16 B] makes the warp's c-th load one
// contiguous 512-byte segment. Thread per 16-byte chunk.
__global__ void k_tile_quarter_rows(const int4* __restrict__ src, int4* __restrict__ dst, int64_t n_rows,
                                    int nch) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n_rows * nch) return;
    const int64_t r = i / nch;
    const int j = (int)(i % nch), cpq = nch / 4;
    const int q = j / cpq, c = j % cpq;
    const int lane = (int)(r & 7) * 4 + q;
    dst[(r >> 3) * 8 * nch + (int64_t)c * 32 + lane] = src[i];
}

// Lane-tiled layout for the Q8_0 gate/up rows: within each row, 16-byte
// chunk (c * 32 + l) holds half (c % 2) of block l + 32 * (c / 2), so lane l
// owns whole blocks and every warp load is contiguous. Thread per chunk.
__global__ void k_tile_block_rows(const int4* __restrict__ src, int4* __restrict__ dst, int64_t n_rows, int nch) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // destination chunk
    if (i >= n_rows * nch) return;
    const int64_t r = i / nch;
    const int n = (int)(i % nch), c = n / 32, l = n % 32;
    dst[i] = src[r * nch + 2 * (l + 32 * (c / 2)) + (c % 2)];
}

}  // namespace

// ===========================================================================
// Host side
// ===========================================================================

static int64_t gguf_bytes(int qtype, int64_t n) {
    if (qtype == PI_QT_Q8_0) return n / 32 * 34;
    if (qtype == PI_QT_Q4_0) return n / 32 * 18;
    if (qtype == PI_QT_F32) return n * 4;
    return -1;
}

int pi_tile_down_mats(pi_ctx* ctx, PiMats* m, std::vector<void*>* allocs) {
    const int64_t row_bytes = m->q_row_bytes();
    if (row_bytes % 64 || m->rows % 8) return pi_set_error(ctx, PI_ERR_ARG, "down tiling: bad shape");
    const int nch = (int)(row_bytes / 16);
    const int64_t n_rows = m->n * m->rows;
    void* dst = nullptr;
    if (pi_cuda_check(ctx, cudaMalloc(&dst, (size_t)(n_rows * row_bytes)), "cudaMalloc(tiled)")) return PI_ERR_OOM;
    k_tile_quarter_rows<<<(unsigned)((n_rows * nch + 255) / 256), 256>>>((const int4*)m->q, (int4*)dst, n_rows, nch);
    if (pi_cuda_check(ctx, cudaDeviceSynchronize(), "tile down")) {
        cudaFree(dst);
        return PI_ERR_CUDA;
    }
    for (auto& p : *allocs)
        if (p == m->q) p = dst;
    cudaFree(m->q);
    m->q = dst;
    return PI_OK;
}

int pi_tile_gateup_mats(pi_ctx* ctx, PiMats* m, std::vector<void*>* allocs) {
    const int64_t row_bytes = m->q_row_bytes();
    if (row_bytes % 1024) return pi_set_error(ctx, PI_ERR_ARG, "gate/up tiling: row must be a multiple of 1024 bytes");
    const int nch = (int)(row_bytes / 16);
    const int64_t n_rows = m->n * m->rows;
    void* dst = nullptr;
    if (pi_cuda_check(ctx, cudaMalloc(&dst, (size_t)(n_rows * row_bytes)), "cudaMalloc(tiled)")) return PI_ERR_OOM;
    k_tile_block_rows<<<(unsigned)((n_rows * nch + 255) / 256), 256>>>((const int4*)m->q, (int4*)dst, n_rows, nch);
    if (pi_cuda_check(ctx, cudaDeviceSynchronize(), "tile gate/up")) {
        cudaFree(dst);
        return PI_ERR_CUDA;
    }
    for (auto& p : *allocs)
        if (p == m->q) p = dst;
    cudaFree(m->q);
    m->q = dst;
    return PI_OK;
}

int pi_repack_mats(pi_ctx* ctx, PiMats* m, const void* raw, int qtype, int64_t n, int64_t rows, int64_t cols,
                   int src_on_host, std::vector<void*>* allocs) {
    m->qtype = qtype;
    m->n = n;
    m->rows = rows;
    m->cols = cols;
    const int64_t per_mat = gguf_bytes(qtype, rows * cols);
    const int64_t qb = m->q_mat_bytes() * n;
    const int64_t nd = m->d_mat_elems() * n;
    if (pi_cuda_check(ctx, cudaMalloc(&m->q, (size_t)qb), "cudaMalloc(weights)")) return PI_ERR_OOM;
    allocs->push_back(m->q);
    if (pi_cuda_check(ctx, cudaMalloc(&m->d, (size_t)nd * 2), "cudaMalloc(scales)")) return PI_ERR_OOM;
    allocs->push_back(m->d);
    // Stage host sources one matrix at a time.
    void* stage = nullptr;
    if (src_on_host) {
        if (pi_cuda_check(ctx, cudaMalloc(&stage, (size_t)per_mat), "cudaMalloc(stage)")) return PI_ERR_OOM;
    }
    const int64_t nblk = rows * cols / 32;
    int rc = PI_OK;
    for (int64_t i = 0; i < n && rc == PI_OK; ++i) {
        const uint8_t* src = (const uint8_t*)raw + i * per_mat;
        if (src_on_host) {
            if (pi_cuda_check(ctx, cudaMemcpy(stage, src, (size_t)per_mat, cudaMemcpyHostToDevice), "upload")) {
                rc = PI_ERR_CUDA;
                break;
            }
            src = (const uint8_t*)stage;
        }
        const int thr = 256;
        const int64_t grid = (nblk + thr - 1) / thr;
        if (qtype == PI_QT_Q8_0)
            k_repack_q8<<<(unsigned)grid, thr>>>(src, nblk, (int8_t*)m->q + i * m->q_mat_bytes(),
                                                  m->d + i * m->d_mat_elems());
        else
            k_repack_q4<<<(unsigned)grid, thr>>>(src, nblk, (uint8_t*)m->q + i * m->q_mat_bytes(),
                                                  m->d + i * m->d_mat_elems());
        if (pi_cuda_check(ctx, cudaGetLastError(), "repack")) rc = PI_ERR_CUDA;
        if (src_on_host && rc == PI_OK && pi_cuda_check(ctx, cudaDeviceSynchronize(), "repack sync"))
            rc = PI_ERR_CUDA;
    }
    if (stage) cudaFree(stage);
    if (rc == PI_OK && pi_cuda_check(ctx, cudaDeviceSynchronize(), "repack")) rc = PI_ERR_CUDA;
    return rc;
}

namespace {
struct FwdBufs {
    float* normed;
    int8_t* xq;
    float* xs;
    float* logits;
    int32_t* flag_list;
    int32_t* n_flag;
    int32_t* idx;
    float* gates;
    float* shscale;
    int32_t* counts;
    int32_t* offsets;
    int32_t* perm;
    int32_t* slot_of;
    int4* items;
    int32_t* n_items;
    int8_t* hq;
    float* hs;
    float* hf;
    float* y;
    __half *xh, *xl, *hh, *hl;
    __half *xth, *xtl;  // tensor-core router: tokens split into f16 hi/lo
    float* xnorm;
    __half* h16;  // Q8_0 prefill GEMM: h in slot order as exact f16
    int32_t* disp_cc;   // large-batch dispatch: per-chunk expert counts
    size_t bytes;
};

// Prefill-sized batches route with the certified tensor-core router (when the
// layer supports it); PI_ROUTER=wide forces the exact SIMT router instead.
bool use_router_tc(const pi_moe_layer* L, int64_t T) {
    static const bool wide = [] {
        const char* v = std::getenv("PI_ROUTER");
        return v && v[0] == 'w';
    }();
    return T >= 256 && L->router_tc && !wide;
}

// Prefill-sized batches take the tensor-core GEMM path (Q4_0 weights). The
// environment variable PI_PREFILL=0/1 forces the choice (tests, benchmarks).
bool use_gemm(const pi_moe_layer* L, int64_t T, int flags) {
    if (L->qtype != PI_QT_Q4_0 && L->qtype != PI_QT_Q8_0) return false;
    if (flags & PI_FWD_FORCE_GEMV) return false;
    if (flags & PI_FWD_FORCE_GEMM) return true;  // PI_ERR_ARG on shapes the GEMM does not tile
    if (L->qtype == PI_QT_Q4_0 ? !pi_prefill_shape_ok(L->d, L->f) : !pi_prefill_q8_shape_ok(L->d, L->f)) return false;
    static const int force = [] {
        const char* v = std::getenv("PI_PREFILL");
        return v ? (v[0] == '1' ? 1 : 0) : -1;
    }();
    if (force >= 0) return force == 1;
    return T >= 128;
}

// Upper bound of the work items k_dispatch writes for item size tg: one partial
// item per used expert plus full ones, and the shared expert's items. The expert
// kernels launch this many CTA rows; rows past the realised count exit at once,
// so the bound is kept tight (each launched CTA occupies an SM while it checks).
int64_t max_items(const pi_moe_layer* L, int64_t T, int tg) {
    const int64_t Tk = T * L->k;
    return std::min<int64_t>(L->E, Tk) + Tk / tg + (L->has_shared ? (T + tg - 1) / tg : 0) + 1;
}

// Dispatch of T tokens x k experts (see k_dispatch): the chunked counting sort for
// large batches (cc: scratch of (ceil(T / DC) + 1) * E ints), the per-expert kernel
// otherwise. n_sh: shared-expert slots (default T); n_routed_dev: see k_disp_scan.
void launch_dispatch(cudaStream_t st, const int32_t* idx, const int32_t* counts, int T, int k, int E, int has_shared,
                     int32_t* offsets, int32_t* perm, int32_t* slot_of, int4* items, int32_t* n_items, int tg,
                     int32_t* cc, int n_sh = -1, int32_t* n_routed_dev = nullptr) {
    if (cc && ((int64_t)T * k >= 4096 || n_routed_dev) && E <= DC_MAXE) {
        const int nchunk = (T + DC - 1) / DC;
        int32_t* offs = offsets ? offsets : cc + (size_t)nchunk * E;  // offsets are needed by the scatter
        k_disp_count<<<(unsigned)nchunk, DC, 0, st>>>(idx, T, k, E, cc);
        k_disp_scan<<<1, 512, 0, st>>>(cc, nchunk, T, k, E, has_shared ? (n_sh >= 0 ? n_sh : T) : 0, tg, offs, items,
                                       n_items, n_routed_dev);
        k_disp_scatter<<<(unsigned)nchunk, DC, 0, st>>>(idx, T, k, E, cc, offs, perm, slot_of);
        return;
    }
    if (T >= 8192)
        k_dispatch<4><<<(unsigned)(E + 1), 256, 0, st>>>(idx, counts, T, k, E, has_shared, offsets, perm, slot_of,
                                                         items, n_items, tg);
    else
        pi_pdl_launch(k_dispatch<1>, dim3((unsigned)(E + 1)), dim3(256), 0, st, idx, counts, T, k, E, has_shared, offsets, perm, slot_of,
                                                         items, n_items, tg);
}

FwdBufs carve(const pi_moe_layer* L, int64_t T, int flags, char* base) {
    PiBump b{base};
    FwdBufs f;
    const int64_t d = L->d, F = L->f, E = L->E, k = L->k;
    const int64_t slots = T * k + (L->has_shared ? T : 0);
    f.normed = b.take<float>(T * d);
    f.xq = b.take<int8_t>(T * d);
    f.xs = b.take<float>(T * (d / 32));
    f.logits = b.take<float>(T * (E + 1));
    f.flag_list = b.take<int32_t>(T);
    f.n_flag = b.take<int32_t>(2 + (T + 7) / 8);  // [0] flagged tokens, [1..] router tickets
    f.idx = b.take<int32_t>(T * k);
    f.gates = b.take<float>(T * k);
    f.shscale = b.take<float>(T);
    f.counts = b.take<int32_t>(E);
    f.offsets = b.take<int32_t>(E);
    f.perm = b.take<int32_t>(T * k);
    f.slot_of = b.take<int32_t>(T * k);
    f.items = b.take<int4>(max_items(L, T, TG));  // TG is the smallest item size
    f.disp_cc = b.take<int32_t>(((T + DC - 1) / DC + 1) * E);
    f.n_items = b.take<int32_t>(1);
    f.hq = b.take<int8_t>(slots * F);
    f.hs = b.take<float>(slots * (F / 32));
    f.hf = b.take<float>(slots * F);
    f.y = b.take<float>(slots * d);
    if (use_gemm(L, T, flags) && L->qtype == PI_QT_Q8_0) {
        f.h16 = b.take<__half>(slots * F);
    } else {
        f.h16 = nullptr;
    }
    if (use_gemm(L, T, flags) && L->qtype == PI_QT_Q4_0) {
        f.xh = f.xl = nullptr;
        f.hh = b.take<__half>(slots * F);
        f.hl = b.take<__half>(slots * F);
    } else {
        f.xh = f.xl = f.hh = f.hl = nullptr;
    }
    if (use_router_tc(L, T) || (use_gemm(L, T, flags) && L->qtype == PI_QT_Q4_0)) {
        f.xth = b.take<__half>(T * d);
        f.xtl = b.take<__half>(T * d);
        f.xnorm = b.take<float>(T);
    } else {
        f.xth = f.xtl = nullptr;
        f.xnorm = nullptr;
    }
    f.bytes = b.off + 256;
    return f;
}
}  // namespace

// Expert kernel arguments for a dispatch over `n_routed` routed slots (then the
// shared expert's slots); item.x == E_items marks the shared expert.
ExpertArgs expert_args(const pi_moe_layer* L, int E_items, const FwdBufs& B, const int32_t* perm, int64_t n_routed,
                       const float* xin) {
    ExpertArgs a;
    a.g = L->gate.q;
    a.u = L->up.q;
    a.dn = L->down.q;
    a.gd = L->gate.d;
    a.ud = L->up.d;
    a.dd = L->down.d;
    a.gs = L->gate_sh.q;
    a.us = L->up_sh.q;
    a.dns = L->down_sh.q;
    a.gsd = L->gate_sh.d;
    a.usd = L->up_sh.d;
    a.dsd = L->down_sh.d;
    a.E = E_items;
    a.d = (int)L->d;
    a.f = (int)L->f;
    a.items = B.items;
    a.n_items = B.n_items;
    a.perm = perm;
    a.n_routed = (int)n_routed;
    a.xq = B.xq;
    a.xs = B.xs;
    a.xf = xin;
    a.hq = B.hq;
    a.hs = B.hs;
    a.hf = B.hf;
    a.y = B.y;
    a.h16 = B.h16;
    a.n_routed_dev = nullptr;
    a.sh_row0 = 0;
    a.n_sh = 0;
    return a;
}

// Expert SwiGLU products of the dispatched work items into a.y (slot order):
// the tensor-core GEMMs for prefill-sized batches, the GEMV kernels otherwise.
// T: token rows behind the slots (Q4_0 GEMM: B.xth/B.xtl hold their f16 split).
int run_experts(pi_ctx* ctx, const pi_moe_layer* L, const ExpertArgs& a, int64_t T, int64_t n_slots, unsigned ni,
                bool gemm, const FwdBufs& B, cudaStream_t st, int flags = 0) {
    const bool q8 = L->qtype == PI_QT_Q8_0;
    const int d = (int)L->d;
    if (gemm && q8) return pi_prefill_experts_q8(ctx, L, a, ni, T, n_slots, flags, st);
    if (gemm) return pi_prefill_experts(ctx, L, a, ni, n_slots, B.xth, B.xtl, T, B.hh, B.hl, st);
    const dim3 gu((unsigned)(L->f / (q8 ? GU_ROWS : 32)), ni), dn((unsigned)(L->d / (q8 ? DN_ROWS : 128)), ni);
    if (q8) {
        {
        PiProfScope ps(ctx, st, "k_gateup");
        switch (d / 512) {
#define GU_Q8(C)                                                                                              \
    case C: {                                                                                                 \
        pi_smem_attr((const void*)k_gateup_q8<C>, gateup_q8_smem<C>());                                       \
        pi_pdl_launch(k_gateup_q8<C>, dim3(gu), dim3(GU_WARPS * 32), gateup_q8_smem<C>(), st, a);                                             \
        break;                                                                                                \
    }
            GU_Q8(2)
            GU_Q8(4)
#undef GU_Q8
            default: return pi_set_error(ctx, PI_ERR_ARG, "Q8_0 layer: n_embd must be 1024 or 2048");
        }
        }
        {
            PiProfScope ps(ctx, st, "k_quant_h");
            const int64_t nblk = n_slots * (L->f / 32);
            pi_pdl_launch(k_quant_h, dim3((unsigned)((nblk * 8 + 255) / 256)), dim3(256), 0, st, B.hf, nblk, B.hq, B.hs);
        }
        PiProfScope ps(ctx, st, "k_down");
        const int cpq = L->f % 64 ? 0 : (int)(L->f / 64);  // 16-byte chunks per quarter row
        if (cpq == 2 || cpq == 4 || cpq == 8) {  // streamed down: persistent CTAs fed by bulk copies
            pi_smem_attr((const void*)k_down_q8s<2>, DSL<2>::SMEM);
            pi_smem_attr((const void*)k_down_q8s<4>, DSL<4>::SMEM);
            pi_smem_attr((const void*)k_down_q8s<8>, DSL<8>::SMEM);
            const unsigned g = (unsigned)std::min<int64_t>((int64_t)ni * (L->d / DS_ROWS), ctx->sm_count);
            switch (cpq) {
                case 2: pi_pdl_launch(k_down_q8s<2>, dim3(g), dim3(DS_THREADS), DSL<2>::SMEM, st, a, ctx->dev_err); break;
                case 4: pi_pdl_launch(k_down_q8s<4>, dim3(g), dim3(DS_THREADS), DSL<4>::SMEM, st, a, ctx->dev_err); break;
                case 8: pi_pdl_launch(k_down_q8s<8>, dim3(g), dim3(DS_THREADS), DSL<8>::SMEM, st, a, ctx->dev_err); break;
            }
            return pi_cuda_check(ctx, cudaGetLastError(), "experts") ? PI_ERR_CUDA : PI_OK;
        }
        // CPQ = 16: term buffer + staged h above the default 48 KB
        pi_smem_attr((const void*)k_down_q8<16>, dn_smem(16));
        if (cpq != 16)  // widths 128, 256, 512 took the streamed kernel above
            return pi_set_error(ctx, PI_ERR_ARG, "Q8_0 layer: expert width must be 128, 256, 512 or 1024");
        k_down_q8<16><<<dn, 256, dn_smem(16), st>>>(a);
    } else {
        {
        PiProfScope ps(ctx, st, "k_gateup");
        switch (d / 1024) {
            case 1: k_gateup_q4<1><<<gu, 512, 0, st>>>(a); break;
            case 2: k_gateup_q4<2><<<gu, 512, 0, st>>>(a); break;
            case 4: k_gateup_q4<4><<<gu, 512, 0, st>>>(a); break;
            default: return pi_set_error(ctx, PI_ERR_ARG, "Q4_0 layer: n_embd must be 1024, 2048 or 4096");
        }
        }
        PiProfScope ps(ctx, st, "k_down");
        switch (L->f / 128) {
            case 1: k_down_q4<1><<<dn, 256, 0, st>>>(a); break;
            case 2: k_down_q4<2><<<dn, 256, 0, st>>>(a); break;
            case 4: k_down_q4<4><<<dn, 256, 0, st>>>(a); break;
            case 8: k_down_q4<8><<<dn, 256, 0, st>>>(a); break;
            default: return pi_set_error(ctx, PI_ERR_ARG, "Q4_0 layer: expert width must be 128..1024 (x2)");
        }
    }
    return pi_cuda_check(ctx, cudaGetLastError(), "experts") ? PI_ERR_CUDA : PI_OK;
}

int pi_router_prepare(pi_ctx* ctx, pi_moe_layer* L) {
    L->ep = (L->E + RW_ROWS - 1) / RW_ROWS * RW_ROWS;
    const size_t bytes = sizeof(float) * (size_t)L->d * L->ep;
    if (pi_cuda_check(ctx, cudaMalloc((void**)&L->router_t, bytes), "cudaMalloc")) return PI_ERR_OOM;
    L->allocs.push_back(L->router_t);
    if (pi_cuda_check(ctx, cudaMemset(L->router_t, 0, bytes), "memset")) return PI_ERR_CUDA;
    const int64_t n = (int64_t)L->E * L->d;
    k_transpose_rows<<<(unsigned)((n + 255) / 256), 256>>>(L->router, L->E, (int)L->d, L->ep, L->router_t);
    if (pi_cuda_check(ctx, cudaDeviceSynchronize(), "router transpose")) return PI_ERR_CUDA;

    // tensor-core router operands: W 2^rs = hi + lo in f16, with max |W| 2^rs in [2^12, 2^13)
    // (no overflow; lo parts of all but tiny elements stay normal); row norms rounded up
    L->router_tc = false;
    if (L->E > 256 || L->E % 16 || L->d % KC_ROUTER || L->E > 32 * TC_PER_LANE) return PI_OK;
    std::vector<float> w((size_t)n);
    if (pi_cuda_check(ctx, cudaMemcpy(w.data(), L->router, sizeof(float) * n, cudaMemcpyDeviceToHost), "router"))
        return PI_ERR_CUDA;
    double amax = 0.0;
    for (float v : w) amax = std::max(amax, (double)std::fabs(v));
    if (!(amax > 0.0) || !std::isfinite(amax)) return PI_OK;
    int ex = 0;
    std::frexp(amax, &ex);  // amax in [2^(ex-1), 2^ex)
    L->router_rs = 13 - ex;
    std::vector<__half> hi((size_t)n), lo((size_t)n);
    std::vector<float> nrm((size_t)L->E);
    for (int64_t e = 0; e < L->E; ++e) {
        double ss = 0.0;
        for (int64_t i = 0; i < L->d; ++i) {
            const size_t j = (size_t)(e * L->d + i);
            const float v = std::ldexp(w[j], L->router_rs);  // exact (power of two, no overflow)
            hi[j] = __float2half_rn(v);
            lo[j] = __float2half_rn(v - __half2float(hi[j]));
            ss += (double)w[j] * (double)w[j];
        }
        nrm[(size_t)e] = (float)(std::sqrt(ss) * (1.0 + 1e-6));  // above the f64 value, which is within 1e-12
    }
    auto up = [&](void** dst, const void* src, size_t b) {
        if (pi_cuda_check(ctx, cudaMalloc(dst, b), "cudaMalloc")) return PI_ERR_OOM;
        L->allocs.push_back(*dst);
        return pi_cuda_check(ctx, cudaMemcpy(*dst, src, b, cudaMemcpyHostToDevice), "router copy") ? PI_ERR_CUDA
                                                                                                      : PI_OK;
    };
    if (int rc = up((void**)&L->router_h, hi.data(), sizeof(__half) * n)) return rc;
    if (int rc = up((void**)&L->router_l, lo.data(), sizeof(__half) * n)) return rc;
    if (int rc = up((void**)&L->router_nrm, nrm.data(), sizeof(float) * L->E)) return rc;
    L->router_tc = pi_router_maps(L);
    return PI_OK;
}

size_t pi_moe_scratch_bytes(const pi_moe_layer* L, int64_t T, int flags) { return carve(L, T, flags, nullptr).bytes; }

int pi_moe_run(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, float* out, int flags, int32_t* idx_out,
               float* gates_out, int32_t* counts_out, int32_t* offsets_out, int32_t* perm_out, char* scratch,
               cudaStream_t st) {
    FwdBufs B = carve(L, T, flags, scratch);
    const int d = (int)L->d, E = L->E, k = L->k;
    const bool q8 = L->qtype == PI_QT_Q8_0;
    const bool route_only = (out == nullptr);
    const int do_norm = (flags & PI_FWD_RMSNORM) ? 1 : 0;
    const float* xin = do_norm ? B.normed : x;
    int32_t* idx = idx_out ? idx_out : B.idx;
    float* gates = gates_out ? gates_out : B.gates;
    int32_t* counts = counts_out ? counts_out : B.counts;
    int32_t* offsets = offsets_out ? offsets_out : B.offsets;
    int32_t* perm = perm_out ? perm_out : B.perm;

    const bool quant = q8 && (!route_only || (flags & PI_FWD_KEEP_Q8));
    if (do_norm || quant) {
        PiProfScope ps(ctx, st, "k_prep");
        const bool split = use_router_tc(L, T);  // the router's hi/lo split comes from this pass
        if (T >= 1024)
            pi_pdl_launch(k_prep<128>, dim3((unsigned)T), dim3(128), sizeof(float) * d, st, x, d, do_norm, 1e-6f,
                          B.normed, quant ? 1 : 0, B.xq, B.xs, split ? B.xth : nullptr, split ? B.xtl : nullptr,
                          split ? B.xnorm : nullptr);
        else
            pi_pdl_launch(k_prep<256>, dim3((unsigned)T), dim3(256), sizeof(float) * d, st, x, d, do_norm, 1e-6f,
                          B.normed, quant ? 1 : 0, B.xq, B.xs, split ? B.xth : nullptr, split ? B.xtl : nullptr,
                          split ? B.xnorm : nullptr);
    }
    // routing: certified fast logits, then exact logits for the tokens that could not be certified
    if (pi_cuda_check(ctx, cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, st), "memset counts")) return PI_ERR_CUDA;
    if (pi_cuda_check(ctx, cudaMemsetAsync(B.n_flag, 0, sizeof(int32_t) * (2 + (T + 7) / 8), st), "memset flags"))
        return PI_ERR_CUDA;
    if (use_router_tc(L, T)) {
        // prefill-sized batch: fast logits on tensor cores, exact chains for the
        // candidates of each token, the exact path for tokens that stay uncertain
        if (!(do_norm || quant)) {  // else k_prep made the split
            PiProfScope ps(ctx, st, "k_split_tokens");
            k_split_tokens<<<(unsigned)T, 256, 0, st>>>(xin, d, B.xth, B.xtl, B.xnorm);
        }
        if (int rc = pi_router_logits_tc(ctx, L, B.xth, B.xtl, T, B.logits, st)) return rc;
        {
            PiProfScope ps(ctx, st, "k_router_cand");
            // tiles of tokens: one CTA per SM where T allows, at most RC_TT tokens each
            const int64_t sms = ctx->sm_count > 0 ? ctx->sm_count : 148;
            const int tt = (int)std::min<int64_t>(RC_TT, std::max<int64_t>(16, (T + sms - 1) / sms));
            pi_smem_attr((const void*)k_router_cand, router_cand_smem());
            k_router_cand<<<(unsigned)((T + tt - 1) / tt), RC_THR, router_cand_smem(), st>>>(
                B.logits, B.xnorm, L->router_nrm, L->router_rs, xin, L->router, L->bias, (int)T, tt, d, E, k,
                L->has_shared_gate ? 1 : 0, idx, gates, B.shscale, counts, B.flag_list, B.n_flag);
        }
        {
            PiProfScope ps(ctx, st, "k_router_exact");
            dim3 eg((unsigned)((E + 1 + 31) / 32), (unsigned)std::min<int64_t>(T, 64));
            pi_smem_attr((const void*)k_router_exact_list, EX_SMEM);
            k_router_exact_list<<<eg, EX_THREADS, EX_SMEM, st>>>(xin, L->router, L->bias, d, E, B.flag_list, B.n_flag,
                                                                 B.logits);
            launch_topk((unsigned)std::min<int64_t>((T + TK_WARPS - 1) / TK_WARPS, 16), st, B.logits, (int)T, E, k, L->has_shared_gate ? 1 : 0, idx, gates, B.shscale, counts, B.flag_list, B.n_flag);
        }
    } else if (T >= 256) {
        // prefill-sized batch: exact logits for every token, exact selection
        {
            PiProfScope ps(ctx, st, "k_router_wide");
            dim3 rg((unsigned)((T + 31) / 32), (unsigned)(L->ep / RW_ROWS));
            k_router_wide<8><<<rg, RW_THREADS, 0, st>>>(xin, L->router_t, L->ep, L->bias,
                                                        L->has_shared_gate ? L->router + (size_t)E * d : nullptr,
                                                        (int)T, d, E, B.logits);
        }
        PiProfScope ps(ctx, st, "k_topk");
        launch_topk((unsigned)std::min<int64_t>((T + TK_WARPS - 1) / TK_WARPS, 8 * ctx->sm_count), st, B.logits, (int)T, E, k, L->has_shared_gate ? 1 : 0, idx, gates, B.shscale, counts, nullptr, nullptr);
    } else if (L->d % 128 == 0 && L->d <= 4096) {
        // decode-sized batch: exact logits of every token, one chain per lane
        {
            PiProfScope ps(ctx, st, "k_router_dec");
            const int hs = L->has_shared_gate ? 1 : 0;
            int32_t* tickets = B.n_flag + 1;
            // small batches: router + top-k in one launch (the last CTA of a token group
            // routes it); larger ones route in a separate launch with a warp per token
            const int fuse = T <= 8 ? 1 : 0;
            if (d <= 2048) {
                // rows per CTA shrink with the batch, so that the CTAs (and the SMs staging
                // router rows) stay many: R rows x TK tokens per 128-thread CTA
#define RDL(R, TK, N)                                                                                         \
    {                                                                                                         \
        dim3 rg((unsigned)((E + 1 + R - 1) / R), (unsigned)((T + TK - 1) / TK));                              \
        pi_smem_attr((const void*)k_router_dec<R, TK, N, true, 128>, rd_smem<R, TK>(2048));                   \
        pi_pdl_launch(k_router_dec<R, TK, N, true, 128>, rg, dim3(128), rd_smem<R, TK>(d), st, xin, L->router, \
                      L->bias, (int)T, d, E, B.logits, k, hs, idx, gates, B.shscale, counts, tickets, fuse,  \
                      ctx->dev_err);                                                                          \
    }
#define RD16(N)                                   \
    {                                             \
        if (T <= 2) RDL(2, 2, N)                  \
        else if (T <= 8) RDL(4, 8, N)             \
        else RDL(16, 8, N)                        \
    }
                if (E <= 64) RD16(2) else if (E <= 128) RD16(4) else if (E <= 256) RD16(8) else RD16(16)
#undef RD16
#undef RDL
                if (!fuse)
                    launch_topk((unsigned)std::min<int64_t>((T + TK_WARPS - 1) / TK_WARPS, 8 * ctx->sm_count), st,
                                B.logits, (int)T, E, k, hs, idx, gates, B.shscale, counts, nullptr, nullptr);
            } else {
                pi_smem_attr((const void*)k_router_dec<8, 4, 16, false, 32>, rd_smem<8, 4>(4096));
                dim3 rg((unsigned)((E + 1 + 7) / 8), (unsigned)((T + 3) / 4));
                pi_pdl_launch(k_router_dec<8, 4, 16, false, 32>, dim3(rg), dim3(32), rd_smem<8, 4>(d), st, 
                    xin, L->router, L->bias, (int)T, d, E, B.logits, k, hs, idx, gates, B.shscale, counts, tickets, 0,
                    ctx->dev_err);
                launch_topk((unsigned)std::min<int64_t>((T + TK_WARPS - 1) / TK_WARPS, 8 * ctx->sm_count), st,
                            B.logits, (int)T, E, k, hs, idx, gates, B.shscale, counts, nullptr, nullptr);
            }
        }
    } else {
        return pi_set_error(ctx, PI_ERR_ARG, "router: n_embd must be a multiple of 128, at most 4096");
    }
    const bool gemm = !route_only && use_gemm(L, T, flags);
    const int tg = gemm ? (q8 ? PI_GEMM_NT_Q8 : PI_GEMM_NT) : TG;
    {
        PiProfScope ps(ctx, st, "k_dispatch");
        launch_dispatch(st, idx, counts, (int)T, k, E, L->has_shared ? 1 : 0, offsets, perm, B.slot_of, B.items,
                        B.n_items, tg, B.disp_cc);
    }
    if (route_only) return pi_cuda_check(ctx, cudaGetLastError(), "route") ? PI_ERR_CUDA : PI_OK;

    const int64_t n_slots = T * k + (L->has_shared ? T : 0);
    ExpertArgs a = expert_args(L, E, B, perm, T * k, xin);
    a.n_sh = L->has_shared ? (int)T : 0;
    const unsigned ni = (unsigned)max_items(L, T, tg);
    if (gemm && !q8 && !use_router_tc(L, T)) {  // the router did not split the tokens
        PiProfScope ps(ctx, st, "k_split_tokens");
        k_split_tokens<<<(unsigned)T, 256, 0, st>>>(xin, d, B.xth, B.xtl, B.xnorm);
    }
    if (int rc = run_experts(ctx, L, a, T, n_slots, ni, gemm, B, st, flags)) return rc;
    PiProfScope ps(ctx, st, "k_combine");
    pi_pdl_launch(k_combine, dim3(dim3((unsigned)T, (unsigned)((d + 1023) / 1024))), dim3(256), 0, st, x, B.y, gates, B.slot_of, B.shscale,
                                                                           nullptr, (int)T, k, d,
                                                                           L->has_shared ? 1 : 0,
                                                                           (flags & PI_FWD_RESIDUAL) ? 1 : 0, out);
    return pi_cuda_check(ctx, cudaGetLastError(), "moe forward") ? PI_ERR_CUDA : PI_OK;
}


int pi_moe_ep_route_run(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, int flags, int world,
                        int32_t* idx, float* gates, float* shscale, int8_t* xq, float* xs, int32_t* send_counts,
                        int8_t* send_xq, float* send_xs, int32_t* send_eid, int32_t* slot_row, char* scratch,
                        cudaStream_t st) {
    // routing only; the Q8_0 activations stay in scratch
    if (int rc = pi_moe_run(ctx, L, x, T, nullptr, flags, idx, gates, nullptr, nullptr, nullptr, scratch, st)) return rc;
    const FwdBufs B = carve(L, T, flags, scratch);
    int32_t* send_tok = reinterpret_cast<int32_t*>(scratch + ((B.bytes + 255) & ~(size_t)255));
    const int d = (int)L->d, k = L->k, n = (int)(T * k), per_rank = L->n_exp;
    const int nchunk = (n + EPC - 1) / EPC;
    int32_t* cc = send_tok + ((n + 63) & ~63);  // [nchunk][world]
    PiProfScope ps(ctx, st, "k_ep_layout");
    k_ep_chunk_count<<<(unsigned)nchunk, EPC, 0, st>>>(idx, n, per_rank, world, cc);
    k_ep_scan<<<1, 1, 0, st>>>(cc, nchunk, world, send_counts);
    k_ep_scatter<<<(unsigned)nchunk, EPC, 0, st>>>(idx, n, k, per_rank, world, cc, send_tok, send_eid, slot_row);
    k_ep_gather<<<(unsigned)n, 128, 0, st>>>(B.xq, B.xs, send_tok, n, d, send_xq, send_xs);
    if (xq && pi_cuda_check(ctx, cudaMemcpyAsync(xq, B.xq, (size_t)T * d, cudaMemcpyDeviceToDevice, st), "xq"))
        return PI_ERR_CUDA;
    if (xs && pi_cuda_check(ctx, cudaMemcpyAsync(xs, B.xs, sizeof(float) * T * (d / 32), cudaMemcpyDeviceToDevice, st),
                            "xs"))
        return PI_ERR_CUDA;
    if (shscale &&
        pi_cuda_check(ctx, cudaMemcpyAsync(shscale, B.shscale, sizeof(float) * T, cudaMemcpyDeviceToDevice, st), "sh"))
        return PI_ERR_CUDA;
    return pi_cuda_check(ctx, cudaGetLastError(), "ep route") ? PI_ERR_CUDA : PI_OK;
}

namespace {
bool rows_gemm(const pi_moe_layer* L, int64_t n_rows) {
    return L->qtype == PI_QT_Q8_0 && pi_prefill_q8_shape_ok(L->d, L->f) && L->maps_ok && n_rows >= 128;
}
}  // namespace

// Scratch of an expert pass over n given rows: one routed slot per row, or (shared
// expert) slots n .. 2n - 1; dispatch arrays and the hidden / output rows only.
FwdBufs carve_rows(const pi_moe_layer* L, int64_t n, char* base) {
    PiBump b{base};
    FwdBufs f{};
    const int64_t d = L->d, F = L->f, slots = 2 * n;
    f.counts = b.take<int32_t>(L->n_exp);
    f.offsets = b.take<int32_t>(L->n_exp);
    f.perm = b.take<int32_t>(n);
    f.slot_of = b.take<int32_t>(n);
    f.items = b.take<int4>(std::min<int64_t>(L->n_exp, n) + 2 * ((n + TG - 1) / TG) + 1);
    f.disp_cc = b.take<int32_t>(((n + DC - 1) / DC + 1) * L->n_exp);
    f.n_items = b.take<int32_t>(1);
    f.hq = b.take<int8_t>(slots * F);
    f.hs = b.take<float>(slots * (F / 32));
    f.hf = b.take<float>(slots * F);
    f.y = b.take<float>(slots * d);
    if (rows_gemm(L, n)) {
        f.h16 = b.take<__half>(slots * F);
    }
    f.bytes = b.off + 256;
    return f;
}

size_t pi_moe_rows_scratch_bytes(const pi_moe_layer* L, int64_t n_rows) { return carve_rows(L, n_rows, nullptr).bytes; }

int pi_moe_rows_run(pi_ctx* ctx, pi_moe_layer* L, int64_t n_rows, const int8_t* xq, const float* xs,
                    const int32_t* eid, float* y, char* scratch, cudaStream_t st) {
    const bool gemm = rows_gemm(L, n_rows), shared_only = eid == nullptr;
    const FwdBufs B = carve_rows(L, n_rows, scratch);
    const int En = L->n_exp, d = (int)L->d, tg = gemm ? PI_GEMM_NT_Q8 : TG;
    if (pi_cuda_check(ctx, cudaMemsetAsync(B.counts, 0, sizeof(int32_t) * En, st), "memset counts")) return PI_ERR_CUDA;
    if (!shared_only) k_ep_hist<<<(unsigned)((n_rows + 255) / 256), 256, 0, st>>>(eid, n_rows, B.counts);
    {
        PiProfScope ps(ctx, st, "k_dispatch");
        // the shared expert alone needs only its items (no routed slots to sort)
        launch_dispatch(st, shared_only ? B.perm : eid, B.counts, (int)n_rows, 1, En, shared_only ? 1 : 0, B.offsets,
                        B.perm, B.slot_of, B.items, B.n_items, tg, shared_only ? nullptr : B.disp_cc);
    }
    ExpertArgs a = expert_args(L, En, B, B.perm, n_rows, nullptr);
    a.n_sh = shared_only ? (int)n_rows : 0;
    a.xq = xq;
    a.xs = xs;
    const int64_t n_slots = shared_only ? 2 * n_rows : n_rows;
    const unsigned ni = (unsigned)(std::min<int64_t>(En, n_rows) + 2 * ((n_rows + tg - 1) / tg) + 1);
    if (int rc = run_experts(ctx, L, a, n_rows, n_slots, ni, gemm, B, st)) return rc;
    k_rows_from_slots<<<(unsigned)n_rows, 256, 0, st>>>(B.y, B.slot_of, n_rows, d, shared_only ? 1 : 0, y);
    return pi_cuda_check(ctx, cudaGetLastError(), "experts") ? PI_ERR_CUDA : PI_OK;
}

int pi_moe_ep_combine_run(pi_ctx* ctx, const pi_moe_layer* L, const float* x, int64_t T, int flags, const float* gates,
                          const float* shscale, const int32_t* slot_row, const float* y_back, const float* y_shared,
                          float* out, cudaStream_t st) {
    const int d = (int)L->d;
    PiProfScope ps(ctx, st, "k_combine");
    pi_pdl_launch(k_combine, dim3(dim3((unsigned)T, (unsigned)((d + 1023) / 1024))), dim3(256), 0, st, 
        x, y_back, gates, slot_row, shscale, y_shared, (int)T, L->k, d, (L->has_shared && y_shared) ? 1 : 0,
        (flags & PI_FWD_RESIDUAL) ? 1 : 0, out);
    return pi_cuda_check(ctx, cudaGetLastError(), "ep combine") ? PI_ERR_CUDA : PI_OK;
}

extern "C" int pi_router_topk_softmax(pi_ctx* ctx, const float* x, int64_t T, const float* router, int64_t d,
                                      int32_t E, int32_t k, int32_t* idx, float* weights, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (T < 0 || E < 1 || E > 512 || k < 1 || k > E || k > 32 || d < 4 || d % 4)
        return pi_set_error(ctx, PI_ERR_ARG, "router: need 1 <= k <= min(E, 32), E <= 512, d % 4 == 0");
    if (T == 0) return PI_OK;
    cudaStream_t st = (cudaStream_t)stream;
    char* scr;
    if (int rc = pi_scratch(ctx, st, (size_t)T * (E + 1) * 4 + 256, &scr)) return rc;
    float* logits = reinterpret_cast<float*>(scr);
    dim3 rg((unsigned)((E + 127) / 128), (unsigned)((T + RT_TT - 1) / RT_TT));
    k_router<<<rg, 128, 0, st>>>(x, router, nullptr, (int)T, (int)d, E, E, logits);
    k_topk_api<<<(unsigned)((T + TK_WARPS - 1) / TK_WARPS), TK_WARPS * 32, 0, st>>>(logits, (int)T, E, k, idx, weights);
    return pi_cuda_check(ctx, cudaGetLastError(), "router") ? PI_ERR_CUDA : PI_OK;
}

// ---------------------------------------------------------------------------
// Expert-parallel passes used by the NVLink data plane (pi_ep.cu).
// ---------------------------------------------------------------------------
namespace {
int ep_home_flags(int flags) {
    return (flags & (PI_FWD_RMSNORM | PI_FWD_RESIDUAL)) | PI_FWD_FORCE_GEMV | PI_FWD_KEEP_Q8;
}

FwdBufs carve_multi(const pi_moe_layer* L, int64_t n_rows, int k, int64_t n_home, char* base) {
    PiBump b{base};
    FwdBufs f{};
    const int64_t d = L->d, F = L->f, En = L->n_exp, nr = n_rows * k, slots = nr + n_home;
    f.offsets = b.take<int32_t>(En);
    f.perm = b.take<int32_t>(nr);
    f.slot_of = b.take<int32_t>(nr);
    f.items = b.take<int4>(En + nr / PI_GEMM_NT_Q8 + n_home / PI_GEMM_NT_Q8 + 4);
    f.n_items = b.take<int32_t>(1);
    f.counts = b.take<int32_t>(1);  // the routed-slot count (device)
    f.disp_cc = b.take<int32_t>(((n_rows + DC - 1) / DC + 1) * En);
    f.hs = b.take<float>(slots * (F / 32));
    f.y = b.take<float>(slots * d);
    f.h16 = b.take<__half>(slots * F);
    f.bytes = b.off + 256;
    return f;
}
}  // namespace

size_t pi_moe_ep_home_bytes(const pi_moe_layer* L, int64_t T, int flags) {
    return pi_moe_scratch_bytes(L, T, ep_home_flags(flags));
}

int pi_moe_ep_home(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, int flags, char* scratch, PiEpHome* H,
                   cudaStream_t st) {
    const int f = ep_home_flags(flags);
    const FwdBufs B = carve(L, T, f, scratch);
    H->idx = B.idx;
    H->gates = B.gates;
    H->shscale = B.shscale;
    H->xq = B.xq;
    H->xs = B.xs;
    if (T == 0) return PI_OK;
    return pi_moe_run(ctx, L, x, T, nullptr, f, nullptr, nullptr, nullptr, nullptr, nullptr, scratch, st);
}

size_t pi_moe_rows_multi_bytes(const pi_moe_layer* L, int64_t n_rows, int k, int64_t n_home) {
    return carve_multi(L, n_rows, k, n_home, nullptr).bytes;
}

int pi_moe_rows_multi_run(pi_ctx* ctx, pi_moe_layer* L, int64_t n_rows, int k, const int8_t* xq, const float* xs,
                          const int32_t* eid, int64_t n_home, const int8_t* xq_home, const float* xs_home, int flags,
                          char* scratch, PiRowsOut* out, cudaStream_t st) {
    if (L->qtype != PI_QT_Q8_0 || !L->maps_ok)
        return pi_set_error(ctx, PI_ERR_ARG, "ep experts: Q8_0 layer of the prefill GEMM shapes");
    const FwdBufs B = carve_multi(L, n_rows, k, n_home, scratch);
    const int En = L->n_exp, tg = PI_GEMM_NT_Q8;
    const int64_t n_sh = L->has_shared ? n_home : 0;
    {
        PiProfScope ps(ctx, st, "k_dispatch");
        launch_dispatch(st, eid, nullptr, (int)n_rows, k, En, n_sh > 0 ? 1 : 0, B.offsets, B.perm, B.slot_of, B.items,
                        B.n_items, tg, B.disp_cc, (int)n_sh, B.counts);
    }
    ExpertArgs a = expert_args(L, En, B, B.perm, 0, nullptr);
    a.xq = xq;
    a.xs = xs;
    a.n_routed_dev = B.counts;
    a.n_sh = (int)n_sh;
    a.xq_sh = xq_home;
    a.xs_sh = xs_home;
    const int64_t n_slots = n_rows * k + n_sh;
    const unsigned ni = (unsigned)(En + n_rows * k / tg + n_sh / tg + 4);
    if (int rc = run_experts(ctx, L, a, n_rows, n_slots, ni, true, B, st, flags)) return rc;
    out->y = B.y;
    out->slot_of = B.slot_of;
    out->n_routed = B.counts;
    return pi_cuda_check(ctx, cudaGetLastError(), "ep experts") ? PI_ERR_CUDA : PI_OK;
}
