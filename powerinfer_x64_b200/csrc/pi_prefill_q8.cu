// Prefill-sized Q8_0 expert products (Q8_0, T = 8192) on the
// tensor cores, bit-exact with the reference.
//
// The reference's Q8_0 matvec (quant/mod.rs:939-957) quantises the activations
// to Q8_0 and sums, block by block in ascending order,
//     acc += (float)sumi_b * (d_w,b * d_x,b),   sumi_b = sum_{k in b} q_w q_x,
// in f32 starting from 0. Here the int8 values of both operands are converted
// exactly to f16 and multiplied with tcgen05.mma kind::f16: every product and
// every partial sum of a block is an integer below 2^20, so the f32 result in
// TMEM is exactly (float)sumi_b. One MMA group per 32-element block writes a
// fresh accumulator into one of DB TMEM buffers; epilogue warps apply the
// block's scales and add it to f32 registers in block order, so each output is
// the reference's own sequence of roundings. The gate/up kernel stacks 64 gate
// rows over the same 64 up rows in one 128-row tile, applies the reference's
// SwiGLU and quantises h to Q8_0 per 32 rows (a warp's 32 lanes), exactly as
// the reference's ffn_swiglu_q does before its down matvec (quant/mod.rs:1184-1249);
// the down kernel writes y.
//
// Warp roles (QT = 672 threads, one CTA per SM):
//   0-15  epilogue: warp w owns TMEM lanes 32 (w % 4) .. +31 (weight rows) and
//         slot columns 32 (w / 4) .. +31;
//   16-19 converters: thread c fetches weight row c and slot row c of block
//         g + RQ - 1 with cp.async, converts block g to f16 tiles (64-byte
//         swizzled K-major) and publishes the block's scales;
//   20    MMA issuer.
// Every mbarrier wait is bounded (1 s) and reports PI_DEVERR_TIMEOUT.
#include "pi_tc.cuh"
// pi_tc.cuh (pi_common.cuh) comes first: it names the quant types that pi_moe.h defines as macros
#include "pi_internal.h"

namespace {
using namespace pitc;

constexpr int QN = PI_GEMM_NT_Q8;  // slots per item (max MMA N)
constexpr int NEPI = 16, NCONV = 4;
constexpr int QT = (NEPI + NCONV + 1) * 32;
constexpr int RQ = 8;              // raw blocks in flight per converter thread
constexpr int TS = 3;              // f16 tile stages
constexpr int DB = 4;              // TMEM block buffers of QN columns
constexpr int TILE = 128 * 64;     // 128 rows x 32 f16
constexpr int RAW = 128 * 32 * 2 + 128 * 4 * 2;  // W and X int8 rows, W scale pair, X scale
constexpr size_t QSMEM = (size_t)RQ * RAW + (size_t)TS * 2 * TILE + 1024;

// 32 int8 (two 16-byte words) -> 32 exact f16 in swizzled row r of a SW64 tile:
// 0x6400 | (b ^ 0x80) is the f16 value 1024 + b + 128, so subtracting 1152 gives b.
PI_DEV void int8_row_to_f16(const uint4 a, const uint4 b, uint8_t* tile, int r) {
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // 16-byte chunk c = elements 8c .. 8c+7
        uint32_t h[4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t v = w[2 * c + j] ^ 0x80808080u;
            const uint32_t lo = __byte_perm(v, 0x64646464u, 0x5140), hi = __byte_perm(v, 0x64646464u, 0x5342);
            const __half2 l2 = __hsub2(*reinterpret_cast<const __half2*>(&lo), off);
            const __half2 h2 = __hsub2(*reinterpret_cast<const __half2*>(&hi), off);
            h[2 * j] = *reinterpret_cast<const uint32_t*>(&l2);
            h[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        *reinterpret_cast<uint4*>(tile + swz(r, c)) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

PI_DEV void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
PI_DEV void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// MODE 0: gate/up (+ SwiGLU, Q8_0 h); MODE 1: down (y).
template <int MODE>
__global__ __launch_bounds__(QT, 1) void k_moe_gemm_q8(ExpertArgs a, uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* tiles = sm;                    // TS stages of {W tile, X tile}
    uint8_t* raws = sm + TS * 2 * TILE;     // RQ stages of raw int8 rows and scales
    __shared__ __align__(8) uint64_t tile_full[TS], tile_free[TS], d_full[DB], d_free[DB], scl_full[DB];
    __shared__ float s_dw[DB][128], s_dx[DB][QN];
    __shared__ uint32_t s_tmem;
    __shared__ int s_row[QN];  // gate/up: token of each slot column; down: slot
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int it = blockIdx.y;
    if (it >= *a.n_items) return;
    const int4 item = a.items[it];
    const bool sh = item.x == a.E;
    const int K = MODE == 0 ? a.d : a.f;
    const int nb = K / 32;
    const int nn = (item.z + 15) & ~15;

    if (tid == 0) {
        for (int i = 0; i < TS; ++i) {
            mbar_init(&tile_full[i], NCONV);
            mbar_init(&tile_free[i], 1);
        }
        for (int i = 0; i < DB; ++i) {
            mbar_init(&d_full[i], 1);
            mbar_init(&d_free[i], NEPI);
            mbar_init(&scl_full[i], NCONV);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int r = tid; r < QN; r += QT) {
        const int sl = item.y + (r < item.z ? r : 0);
        s_row[r] = MODE == 1 ? sl : (sl < a.n_routed ? a.perm[sl] : sl - a.n_routed);
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(DB * QN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ok = true;

    if (warp >= NEPI && warp < NEPI + NCONV) {
        // ---- converters: thread c owns weight row c and slot row c ----
        const int c = tid - NEPI * 32;
        const size_t mat = sh ? 0 : (size_t)item.x * (MODE == 0 ? a.f : a.d);
        const int8_t* wq;
        const __half* wd;
        int wr;  // row within the family (all experts)
        if (MODE == 0) {
            const bool up = c >= 64;
            wq = (const int8_t*)(up ? (sh ? a.us : a.u) : (sh ? a.gs : a.g));
            wd = up ? (sh ? a.usd : a.ud) : (sh ? a.gsd : a.gd);
            wr = (int)mat + blockIdx.x * 64 + (c & 63);
        } else {
            wq = (const int8_t*)(sh ? a.dns : a.dn);
            wd = sh ? a.dsd : a.dd;
            wr = (int)mat + blockIdx.x * 128 + c;
        }
        const int xrow = s_row[c];
        auto issue = [&](int g) {
            uint8_t* rs = raws + (g % RQ) * RAW;
            const int8_t* p0;
            const int8_t* p1;
            if (MODE == 0) {
                // lane-tiled gate/up rows: half h of block B at ((B/32)*64 + h*32 + B%32) * 16 bytes
                const int8_t* row = wq + (size_t)wr * a.d;
                p0 = row + (size_t)((g >> 5) * 64 + (g & 31)) * 16;
                p1 = p0 + 512;
            } else {
                // lane-tiled down rows: 16-byte chunk j of row r at ((r/8)*8*nch + (j%cpq)*32 + (r%8)*4 + j/cpq) * 16
                const int nch = a.f / 16, cpq = nch / 4, j = 2 * g;
                const size_t base = (size_t)(wr >> 3) * 8 * nch + (size_t)(wr & 7) * 4 + j / cpq;
                p0 = wq + (base + (size_t)(j % cpq) * 32) * 16;
                p1 = wq + (base + (size_t)(j % cpq + 1) * 32) * 16;
            }
            cp_async16(rs + c * 32, p0);
            cp_async16(rs + c * 32 + 16, p1);
            cp_async4(rs + 2 * 128 * 32 + c * 4, wd + (size_t)wr * nb + (g & ~1));  // scale pair
            if (MODE == 0) {
                const int8_t* xr = a.xq + (size_t)xrow * a.d + g * 32;
                cp_async16(rs + 128 * 32 + c * 32, xr);
                cp_async16(rs + 128 * 32 + c * 32 + 16, xr + 16);
                cp_async4(rs + 2 * 128 * 32 + 512 + c * 4, a.xs + (size_t)xrow * nb + g);
            } else {
                const int8_t* hr = a.hq + (size_t)xrow * a.f + g * 32;
                cp_async16(rs + 128 * 32 + c * 32, hr);
                cp_async16(rs + 128 * 32 + c * 32 + 16, hr + 16);
                cp_async4(rs + 2 * 128 * 32 + 512 + c * 4, a.hs + (size_t)xrow * nb + g);
            }
        };
        for (int g = 0; g < RQ - 1 && g < nb; ++g) {
            issue(g);
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        for (int g = 0; g < nb; ++g) {
            if (g + RQ - 1 < nb) issue(g + RQ - 1);
            asm volatile("cp.async.commit_group;" ::: "memory");
            asm volatile("cp.async.wait_group %0;" ::"n"(RQ - 1) : "memory");
            const int ts = g % TS, db = g % DB;
            if (g >= TS && !mbar_wait(&tile_free[ts], (g / TS - 1) & 1)) { ok = false; break; }
            if (g >= DB && !mbar_wait(&d_free[db], (g / DB - 1) & 1)) { ok = false; break; }
            const uint8_t* rs = raws + (g % RQ) * RAW;
            uint8_t* wt = tiles + ts * 2 * TILE;
            int8_row_to_f16(*reinterpret_cast<const uint4*>(rs + c * 32), *reinterpret_cast<const uint4*>(rs + c * 32 + 16),
                            wt, c);
            int8_row_to_f16(*reinterpret_cast<const uint4*>(rs + 128 * 32 + c * 32),
                            *reinterpret_cast<const uint4*>(rs + 128 * 32 + c * 32 + 16), wt + TILE, c);
            const __half2 dpair = *reinterpret_cast<const __half2*>(rs + 2 * 128 * 32 + c * 4);
            s_dw[db][c] = __half2float((g & 1) ? __high2half(dpair) : __low2half(dpair));
            s_dx[db][c] = *reinterpret_cast<const float*>(rs + 2 * 128 * 32 + 512 + c * 4);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tile_full[ts]);
                mbar_arrive(&scl_full[db]);
            }
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
    } else if (warp == NEPI + NCONV) {
        // ---- MMA issuer ----
        if (lane == 0) {
            const uint32_t id = idesc(nn);
            for (int g = 0; g < nb; ++g) {
                const int ts = g % TS, db = g % DB;
                if (!mbar_wait(&tile_full[ts], (g / TS) & 1) ||
                    (g >= DB && !mbar_wait(&d_free[db], (g / DB - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint8_t* wt = tiles + ts * 2 * TILE;
                const uint32_t dcol = tmem + db * QN;
                mma_f16(dcol, umma_desc(wt, 0), umma_desc(wt + TILE, 0), id, 0u);
                mma_f16(dcol, umma_desc(wt, 32), umma_desc(wt + TILE, 32), id, 1u);
                mma_commit(&tile_free[ts]);
                mma_commit(&d_full[db]);
            }
        }
    } else {
        // ---- epilogue: rows 32 (w % 4) + lane, slot columns 32 (w / 4) .. +31 ----
        const int q = warp & 3, cg = warp >> 2, rl = 32 * q + lane;
        const bool live = 32 * cg < item.z;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
        for (int g = 0; g < nb; ++g) {
            const int db = g % DB;
            if (!mbar_wait(&d_full[db], (g / DB) & 1) || !mbar_wait(&scl_full[db], (g / DB) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (live) {
                float v[32];
                tmem_ld32(tmem + lane_base + db * QN + 32 * cg, v);
                const float dw = s_dw[db][rl];
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[j] = fadd(acc[j], fmul(v[j], fmul(dw, s_dx[db][32 * cg + j])));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_free[db]);
        }
        if (MODE == 0) {
            // up rows (quarters 2, 3) hand their sums to the gate rows through shared memory
            float* s_up = reinterpret_cast<float*>(raws);  // the raw ring is idle now
            asm volatile("bar.sync 1, %0;" ::"n"(NEPI * 32) : "memory");
            if (q >= 2 && live) {
#pragma unroll
                for (int j = 0; j < 32; ++j) s_up[(32 * (q - 2) + lane) * (QN + 1) + 32 * cg + j] = acc[j];
            }
            asm volatile("bar.sync 1, %0;" ::"n"(NEPI * 32) : "memory");
            if (q < 2 && live) {
                const int f0 = blockIdx.x * 64 + 32 * q;  // first h row of this warp = one Q8_0 block
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int col = 32 * cg + j;
                    if (col < item.z) {  // warp-uniform
                        const float h = swiglu_ref(acc[j], s_up[rl * (QN + 1) + col]);
                        float sc;
                        const int8_t hq = warp_quant_q8(h, &sc);
                        const size_t slot = (size_t)item.y + col;
                        a.hq[slot * a.f + f0 + lane] = hq;
                        if (lane == 0) a.hs[slot * (a.f / 32) + f0 / 32] = sc;
                    }
                }
            }
        } else if (live) {
            const int row = blockIdx.x * 128 + rl;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (32 * cg + j < item.z) a.y[(size_t)(item.y + 32 * cg + j) * a.d + row] = acc[j];
        }
    }
    if (!ok) atomicOr(err, PI_DEVERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(DB * QN) : "memory");
}

}  // namespace

bool pi_prefill_q8_shape_ok(int64_t d, int64_t f) { return d % 1024 == 0 && f % 64 == 0 && d % 128 == 0; }

int pi_prefill_experts_q8(pi_ctx* ctx, const pi_moe_layer* L, const ExpertArgs& a, int64_t max_items,
                          cudaStream_t st) {
    if (L->qtype != PI_QT_Q8_0) return pi_set_error(ctx, PI_ERR_ARG, "prefill Q8_0 GEMM: Q8_0 weights only");
    if (!pi_prefill_q8_shape_ok(a.d, a.f) || (L->has_shared && L->f_sh != L->f))
        return pi_set_error(ctx, PI_ERR_ARG,
                            "prefill Q8_0 GEMM: n_embd must be a multiple of 1024, expert widths equal and a multiple of 64");
    static_assert((size_t)RQ * RAW >= (size_t)64 * (QN + 1) * 4, "the up-row exchange fits in the raw ring");
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_moe_gemm_q8<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QSMEM);
        cudaFuncSetAttribute(k_moe_gemm_q8<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QSMEM);
        attr = true;
    }
    {
        PiProfScope ps(ctx, st, "k_gemm_q8_gateup");
        k_moe_gemm_q8<0><<<dim3((unsigned)(a.f / 64), (unsigned)max_items), QT, QSMEM, st>>>(a, ctx->dev_err);
    }
    {
        PiProfScope ps(ctx, st, "k_gemm_q8_down");
        k_moe_gemm_q8<1><<<dim3((unsigned)(a.d / 128), (unsigned)max_items), QT, QSMEM, st>>>(a, ctx->dev_err);
    }
    return pi_cuda_check(ctx, cudaGetLastError(), "prefill Q8_0 GEMM") ? PI_ERR_CUDA : PI_OK;
}
