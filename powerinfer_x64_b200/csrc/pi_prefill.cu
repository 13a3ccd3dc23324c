// Prefill-sized expert products (Q4_0, T = 512..4096) on the
// 5th-generation tensor cores: tcgen05.mma kind::f16 with f32 accumulators in
// tensor memory (TMEM).
//
// The reference computes Q4_0 expert products as f32 dots of f32 activations
// with dequantised weights (quant/mod.rs:958-969). One f16 pass (weights,
// activations and h rounded to f16) gives ~5e-4 relative L2 but exceeds the
// 2e-3 max-abs bar, and a Q4_0 block's scale is a per-row f16 that cannot be
// factored out of the K sum. So every operand is split into f16 hi + lo parts
// (v = hi + lo, lo = f16(v - hi)) and each k-step issues three MMAs,
//     D += W_hi X_hi + W_lo X_hi + W_hi X_lo,
// which keeps the products within ~2^-21 relative of the f32 result.
//
// Work item: (expert e, <= 256 slots of e); a CTA takes one item and one (gate/up)
// or four (down) 128-row m-tiles of the expert, walking K in 32-element chunks
// (one Q4_0 block per row). MMA N is the item's slot count rounded up to 16.
// Data movement is asynchronous throughout (TMA, no multicast):
//   * raw Q4_0 nibbles [128 rows][16 B] per chunk and f16 scales [128 rows][8]
//     per 8 chunks land in a ring (both weight layouts -- plain rows and the
//     decode kernels' lane-tiled down rows -- are described as tensor maps);
//   * converter warps dequantise them into f16 hi/lo tiles in the canonical
//     K-major 64-byte-swizzled UMMA layout;
//   * the activations (already split into f16 hi/lo, slot-major) are loaded by
//     TMA straight into that layout;
//   * one thread issues the MMAs; tcgen05.commit releases stages and slots.
// The epilogue reads the accumulators with tcgen05.ld (warp w owns TMEM lanes
// 32(w%4)..+31, one weight row per thread) and writes SwiGLU h as f16 hi/lo
// (gate/up) or y (down). All mbarrier waits are bounded (1 s) and report
// PI_DEVERR_TIMEOUT.
#include "pi_tc.cuh"
// pi_tc.cuh (pi_common.cuh) comes first: it names the quant types that pi_moe.h defines as macros
#include "pi_internal.h"

namespace {
using namespace pitc;

constexpr int NTMAX = PI_GEMM_NT;  // slots per item (max MMA N)
constexpr int MT = 128;            // weight rows per m-tile (MMA M)
constexpr int KC = 32;             // K elements per chunk (one 64-byte swizzle atom row)
constexpr int WTILE = MT * 64;     // 128 rows x 64 bytes
constexpr int XTILE = NTMAX * 64;  // 256 rows x 64 bytes
constexpr int RAWQ = MT * 16;      // raw nibbles of one matrix per chunk
constexpr int RAWD = MT * 16;      // raw scales of one matrix per 8 chunks

// 16 elements of one Q4_0 block (8 nibble bytes: part p = 0/1 of the block)
// -> swizzled 16-byte chunks 2p, 2p+1 of row r in the hi and lo tiles.
// Packed f16 arithmetic: 0x6400 | n is the f16 value 1024 + n, so (0x6400 | n) - 1032 = n - 8
// exactly; hi = rn(d * (n - 8)) is one rounding of the exact product, the same value as
// rounding the f32 product (exact: 11 x 4 bits); lo = rn(d * (n - 8) - hi) by one fused
// multiply-add, the same value as rounding the exact f32 difference.
PI_DEV void dequant_part_q4(const uint2 nib, __half sc, uint8_t* th, uint8_t* tl, int r, int p) {
    const uint32_t w[2] = {nib.x, nib.y};
    const __half2 d2 = __half2half2(sc);
    const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6408));  // 1032
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const uint32_t v = w[cc];
        // t_j holds nibble j (bits 0..3) and nibble j + 4 (bits 16..19): elements j, j + 4
        uint32_t t[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) t[j] = (v >> (4 * j)) & 0x000F000Fu;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            // pair q = elements (2q, 2q + 1): low halves of t[2q], t[2q+1] for q < 2, high halves after
            const uint32_t a = t[(2 * q) & 3], b = t[(2 * q + 1) & 3];
            const uint32_t u = (q < 2 ? __byte_perm(a, b, 0x5410) : __byte_perm(a, b, 0x7632)) | 0x64006400u;
            const __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&u), off);
            const __half2 hv = __hmul2(d2, qv);
            const __half2 lv = __hfma2(d2, qv, __hneg2(hv));
            hi[q] = *reinterpret_cast<const uint32_t*>(&hv);
            lo[q] = *reinterpret_cast<const uint32_t*>(&lv);
        }
        *reinterpret_cast<uint4*>(th + swz(r, 2 * p + cc)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(tl + swz(r, 2 * p + cc)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// Warp roles (GT = 352 threads):
//   0-7  converters: dequantise chunk g's raw nibbles into weight stage g % WS,
//        then arrive on the stage's `full` barrier and release the raw slot;
//        after the last chunk of an m-tile they run its epilogue;
//   8    activation producer: TMA of the hi/lo activation chunk into slot g % XS;
//   9    MMA issuer: waits for a weight stage and its activation slot, issues
//        3 x (K/16) MMAs per matrix and releases both with tcgen05.commit;
//   10   weight producer: TMA of raw nibbles (and every 8 chunks the scales)
//        into raw slot g % RS.
constexpr int GT = 352;
constexpr int WS = 3;
constexpr int GU_MPC = 1, DN_MPC = 4;  // 128-row m-tiles handled by one CTA (gate/up, down)
template <int MODE>
constexpr int xs_depth() { return MODE == 0 ? 3 : 4; }  // activation slots
template <int MODE>
constexpr int rs_depth() { return MODE == 0 ? 4 : 8; }  // raw weight slots (<= 9, see the weight producer)
template <int MODE>
constexpr size_t gemm_smem() {
    constexpr int NMAT = MODE == 0 ? 2 : 1;
    static_assert(rs_depth<MODE>() <= 9, "scale slot reuse");
    return (size_t)WS * 2 * NMAT * WTILE + (size_t)xs_depth<MODE>() * 2 * XTILE + (size_t)rs_depth<MODE>() * NMAT * RAWQ +
           (size_t)2 * NMAT * RAWD + 1024;
}

template <int MODE>
__global__ __launch_bounds__(GT, 1) void k_moe_gemm(ExpertArgs a, const __grid_constant__ PiPrefillMaps wm,
                                                    const __grid_constant__ CUtensorMap map_hi,
                                                    const __grid_constant__ CUtensorMap map_lo,
                                                    const __half* __restrict__ xth, const __half* __restrict__ xtl,
                                                    __half* __restrict__ hh, __half* __restrict__ hl, uint32_t* err) {
    constexpr int NMAT = MODE == 0 ? 2 : 1;  // weight matrices per item
    constexpr int XS = xs_depth<MODE>(), RS = rs_depth<MODE>();
    constexpr int WSTAGE = 2 * NMAT * WTILE;  // W hi/lo per matrix
    constexpr uint32_t TCOLS = MODE == 0 ? 512 : 256;
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* xring = sm + WS * WSTAGE;             // XS slots of {hi, lo} activation tiles
    uint8_t* qring = xring + XS * 2 * XTILE;       // RS slots of raw nibbles [NMAT][128][16]
    uint8_t* dring = qring + RS * NMAT * RAWQ;     // 2 slots of raw scales [NMAT][128][8 x f16]
    __shared__ __align__(8) uint64_t wfree[WS], full[WS], xfull[XS], xempty[XS], qfull[RS], qempty[RS];
    __shared__ uint32_t s_tmem;
    __shared__ int s_tok[MODE == 0 ? NTMAX : 1];  // gate/up: token of each slot row
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int it = blockIdx.y;
    if (it >= *a.n_items) return;
    const int4 item = a.items[it];
    const bool sh = item.x == a.E;
    constexpr int mpc = MODE == 0 ? GU_MPC : DN_MPC;  // m-tiles per CTA
    const int row0 = blockIdx.x * mpc * MT;
    const int K = MODE == 0 ? a.d : a.f;
    const int nchunks = K / KC;
    const int n_iter = mpc * nchunks;
    const int nn = (item.z + 15) & ~15;  // MMA N

    if (tid == 0) {
        for (int i = 0; i < WS; ++i) {
            mbar_init(&wfree[i], 1);
            mbar_init(&full[i], 8);  // one arrival per converter warp
        }
        for (int i = 0; i < XS; ++i) {
            mbar_init(&xfull[i], MODE == 0 ? 8 : 1);  // gate/up: one arrival per converter warp
            mbar_init(&xempty[i], 1);
        }
        for (int i = 0; i < RS; ++i) {
            mbar_init(&qfull[i], 1);
            mbar_init(&qempty[i], 8);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ok = true;

    if (warp == 8) {
        // down: activation producer, the slot-major h rows of chunk g as one TMA tile into
        // slot g % XS once the MMAs of chunk g - XS are done (gate/up: the converters gather)
        if (MODE == 1 && lane == 0) {
            for (int g = 0; g < n_iter; ++g) {
                const int slot = g % XS, use = g / XS;
                if (use > 0 && !mbar_wait(&xempty[slot], (use - 1) & 1)) { ok = false; break; }
                uint8_t* xt = xring + slot * 2 * XTILE;
                mbar_expect_tx(&xfull[slot], 2 * XTILE);
                const int xc = (g % nchunks) * KC;
                tma_load_2d(xt, &map_hi, xc, item.y, &xfull[slot]);
                tma_load_2d(xt + XTILE, &map_lo, xc, item.y, &xfull[slot]);
            }
        }
    } else if (warp == 10) {
        // weight producer: raw nibbles of chunk g -> slot g % RS once the converters
        // released chunk g - RS; scales of chunks 8j..8j+7 with chunk 8j into scale slot
        // j % 2, last read by chunks 8j-16..8j-9 -- released in order before chunk
        // 8j - RS, which this wait covers, because RS <= 9)
        if (lane == 0) {
            const int rb = sh ? 0 : item.x * (MODE == 0 ? a.f : a.d);  // expert's first row
            for (int g = 0; g < n_iter; ++g) {
                const int slot = g % RS, use = g / RS, mi = g / nchunks, c = g % nchunks;
                if (use > 0 && !mbar_wait(&qempty[slot], (use - 1) & 1)) { ok = false; break; }
                const bool scales = (c & 7) == 0;
                mbar_expect_tx(&qfull[slot], NMAT * RAWQ + (scales ? NMAT * RAWD : 0));
                const int r0 = rb + row0 + mi * MT;
                uint8_t* qt = qring + slot * NMAT * RAWQ;
                uint8_t* dt = dring + ((g >> 3) & 1) * NMAT * RAWD;
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const int w = MODE == 0 ? m : 2;  // gate, up, down
                    const CUtensorMap* mq = sh ? &wm.q[1][w] : &wm.q[0][w];
                    const CUtensorMap* md = sh ? &wm.d[1][w] : &wm.d[0][w];
                    if (MODE == 0) {
                        tma_load_2d(qt + m * RAWQ, mq, c * 16, r0, &qfull[slot]);
                    } else {
                        // lane-tiled rows: block c of row r at ((r/8)*8*nch + (c % cpq)*32 + (r%8)*4 + c/cpq) * 16 B
                        const int cpq = nchunks / 4;
                        tma_load_4d(qt + m * RAWQ, mq, (c / cpq) * 16, 0, c % cpq, r0 >> 3, &qfull[slot]);
                    }
                    if (scales) tma_load_2d(dt + m * RAWD, md, c, r0, &qfull[slot]);
                }
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            const uint32_t id = idesc(nn);
            for (int g = 0; g < n_iter; ++g) {
                const int s = g % WS, slot = g % XS, c = g % nchunks;
                if (!mbar_wait(&full[s], (g / WS) & 1) || !mbar_wait(&xfull[slot], (g / XS) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint8_t* st = sm + s * WSTAGE;
                const uint8_t* xt = xring + slot * 2 * XTILE;
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const uint8_t* wh = st + 2 * m * WTILE;
                    const uint8_t* wl = wh + WTILE;
                    const uint32_t dcol = tmem + m * NTMAX;
#pragma unroll
                    for (int k = 0; k < KC / 16; ++k) {
                        const uint64_t dwh = umma_desc(wh, 32 * k), dwl = umma_desc(wl, 32 * k);
                        const uint64_t dxh = umma_desc(xt, 32 * k), dxl = umma_desc(xt + XTILE, 32 * k);
                        mma_f16(dcol, dwh, dxh, id, (c > 0 || k > 0) ? 1u : 0u);
                        mma_f16(dcol, dwl, dxh, id, 1u);
                        mma_f16(dcol, dwh, dxl, id, 1u);
                    }
                }
                mma_commit(&wfree[s]);
                mma_commit(&xempty[slot]);
            }
        }
    } else {
        // converter thread t: row r = t / 2, elements 16p .. 16p+15 (p = t % 2) of the chunk's block
        const int r = tid >> 1, p = tid & 1;
        if (MODE == 0) {
            for (int rr = tid; rr < nn; rr += 256) {
                const int sl = item.y + (rr < item.z ? rr : 0);
                s_tok[rr] = sl < a.n_routed ? a.perm[sl] : sl - a.n_routed;
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");
        }
        // gate/up activations: the converters gather chunk g's token rows (16-byte cp.async
        // per row piece, one commit group per chunk) into slot g % XS and publish it one
        // chunk later (wait_group, proxy fence, one arrival per warp); the last chunk at once
        auto publish = [&](int gx) {
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&xfull[gx % XS]);
        };
        for (int g = 0; g < n_iter; ++g) {
            const int s = g % WS, slot = g % RS, mi = g / nchunks, c = g % nchunks;
            if (MODE == 0) {
                const int xs_ = g % XS, xuse = g / XS;
                if (xuse > 0 && !mbar_wait(&xempty[xs_], (xuse - 1) & 1)) { ok = false; break; }
                uint8_t* xt = xring + xs_ * 2 * XTILE;
                for (int q = tid; q < nn * 4; q += 256) {
                    const int row = q >> 2, pc = q & 3;
                    const size_t off = (size_t)s_tok[row] * a.d + c * KC + 8 * pc;
                    const uint32_t dh = smem_u32(xt + swz(row, pc));
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dh), "l"(xth + off) : "memory");
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dh + XTILE), "l"(xtl + off) : "memory");
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
                if (g + 1 < n_iter) {
                    if (g >= 1) {
                        asm volatile("cp.async.wait_group 1;" ::: "memory");
                        publish(g - 1);
                    }
                } else {
                    asm volatile("cp.async.wait_group 0;" ::: "memory");
                    if (g >= 1) publish(g - 1);
                    publish(g);
                }
            }
            if (!mbar_wait(&qfull[slot], (g / RS) & 1)) { ok = false; break; }
            const uint8_t* qt = qring + slot * NMAT * RAWQ;
            const uint8_t* dt = dring + ((g >> 3) & 1) * NMAT * RAWD;
            uint2 nib[NMAT];
            __half sc[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                nib[m] = *reinterpret_cast<const uint2*>(qt + m * RAWQ + r * 16 + 8 * p);
                sc[m] = *reinterpret_cast<const __half*>(dt + m * RAWD + r * 16 + (c & 7) * 2);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&qempty[slot]);
            if (g >= WS && !mbar_wait(&wfree[s], ((g - WS) / WS) & 1)) { ok = false; break; }
            uint8_t* st = sm + s * WSTAGE;
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
                dequant_part_q4(nib[m], sc[m], st + 2 * m * WTILE, st + (2 * m + 1) * WTILE, r, p);
            fence_async_smem();
            tc_fence_before();  // orders this warp's earlier TMEM reads (epilogue) before the next MMAs
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
            if (c + 1 < nchunks) continue;
            // last chunk of m-tile mi: wait for its MMAs, then the epilogue. The next
            // m-tile's first MMA (issued once every converter warp has arrived on the next
            // stage, i.e. after this epilogue) overwrites TMEM.
            if (!mbar_wait(&wfree[s], (g / WS) & 1)) { ok = false; break; }
            tc_fence_after();
            // TMEM lane (warp % 4) * 32 + lane = weight row; warp / 4 takes slot columns [128 (warp / 4), +128)
            const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
            const int row = row0 + mi * MT + (warp & 3) * 32 + lane;
            const int c0 = (warp >> 2) * (NTMAX / 2);
            for (int cb = c0; cb < c0 + NTMAX / 2; cb += 32) {
                if (cb >= item.z) break;
                float gv[32];
                tmem_ld32(tmem + lane_base + cb, gv);
                if (MODE == 0) {
                    float u[32];
                    tmem_ld32(tmem + lane_base + NTMAX + cb, u);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (cb + j < item.z) {
                            const float hvv = gv[j] / (1.0f + __expf(-gv[j])) * u[j];  // tolerance path
                            const __half h1 = __float2half_rn(hvv);
                            const size_t o = (size_t)(item.y + cb + j) * a.f + row;
                            hh[o] = h1;
                            hl[o] = __float2half_rn(hvv - __half2float(h1));
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (cb + j < item.z) a.y[(size_t)(item.y + cb + j) * a.d + row] = gv[j];
                }
            }
            tc_fence_before();
        }
    }
    if (!ok) atomicOr(err, PI_DEVERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
}

// f16 [rows][cols] row-major activations, box {32 columns, 256 rows}, 64-byte
// swizzle (the UMMA K-major SW64 layout); rows past the end read as zeros
bool act_map(CUtensorMap* m, const __half* base, int64_t rows, int64_t cols) {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(__half)};
    const cuuint32_t box[2] = {(cuuint32_t)KC, (cuuint32_t)NTMAX};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}

// Raw Q4_0 nibbles of a plain family [rows][K/2] (box: 16 bytes x 128 rows) and
// the f16 scales [rows][K/32] of any family (box: 8 scales x 128 rows).
bool plain_q_map(CUtensorMap* m, const PiMats& w) {
    const int64_t rows = w.n * w.rows;
    const cuuint64_t dims[2] = {(cuuint64_t)(w.cols / 2), (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(w.cols / 2)};
    const cuuint32_t box[2] = {16, (cuuint32_t)MT};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}
bool scale_map(CUtensorMap* m, const PiMats& w) {
    const int64_t rows = w.n * w.rows;
    const cuuint64_t dims[2] = {(cuuint64_t)(w.cols / 32), (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(w.cols / 32) * sizeof(__half)};
    const cuuint32_t box[2] = {8, (cuuint32_t)MT};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w.d, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}
// Lane-tiled down rows (pi_tile_down_mats): 16-byte block j of row r at
// ((r/8)*8*nch + (j % cpq)*32 + (r%8)*4 + j/cpq) * 16, nch = K/32, cpq = nch/4, as
// a 4-D byte tensor {64 (j/cpq, byte), 8 (r%8), cpq (j%cpq), rows/8 (r/8)}; the box
// {16, 8, 1, 16} is block j of 128 consecutive rows, landing as [128 rows][16 B].
bool tiled_q_map(CUtensorMap* m, const PiMats& w) {
    const int64_t rows = w.n * w.rows, nch = w.cols / 32, cpq = nch / 4;
    const cuuint64_t dims[4] = {64, 8, (cuuint64_t)cpq, (cuuint64_t)(rows / 8)};
    const cuuint64_t strides[3] = {64, 512, (cuuint64_t)(8 * nch * 16)};
    const cuuint32_t box[4] = {16, 8, 1, (cuuint32_t)(MT / 8)};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, w.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// ---------------------------------------------------------------------------
// k_router_gemm: fast router logits for prefill batches. A = tokens [128][K],
// B = router rows [NR][K] (scaled by 2^rs), both split into f16 hi/lo and
// streamed by TMA (K-major SW64, 32-K chunks) through an RG-deep ring.
// Two accumulators keep the error analysis simple: Dh = sum Ah Bh, and
// Dl = sum (Al Bh + Ah Bl), whose terms are ~2^-11 smaller; the logit is
// (Dh + Dl) 2^-rs + bias. Warp 0 loads, warp 1 issues MMAs, warps 2-5 read
// TMEM (warp w: lanes 32 (w % 4) .. +31 = tokens) and store the logits.
// grid (ceil(T / 128), E / NR).
// ---------------------------------------------------------------------------
constexpr int RG = 4;
__global__ __launch_bounds__(192, 1) void k_router_gemm(const __grid_constant__ CUtensorMap mxh,
                                                        const __grid_constant__ CUtensorMap mxl,
                                                        const __grid_constant__ CUtensorMap mwh,
                                                        const __grid_constant__ CUtensorMap mwl, int T, int d, int E,
                                                        int nr, float unscale, const float* __restrict__ bias,
                                                        float* __restrict__ logits, uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
    const int stage = 2 * (MT + nr) * 64;  // A hi/lo + B hi/lo
    __shared__ __align__(8) uint64_t full[RG], empty[RG], done;
    __shared__ uint32_t s_tmem;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * MT, e0 = blockIdx.y * nr;
    const int nchunks = d / KC;
    const uint32_t tcols = nr <= 64 ? 128 : (nr <= 128 ? 256 : 512);
    if (tid == 0) {
        for (int i = 0; i < RG; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ok = true;
    if (warp == 0) {
        if (lane == 0) {
            for (int c = 0; c < nchunks; ++c) {
                const int slot = c % RG, use = c / RG;
                if (use > 0 && !mbar_wait(&empty[slot], (use - 1) & 1)) { ok = false; break; }
                uint8_t* st = sm + slot * stage;
                mbar_expect_tx(&full[slot], stage);
                tma_load_2d(st, &mxh, c * KC, t0, &full[slot]);
                tma_load_2d(st + MT * 64, &mxl, c * KC, t0, &full[slot]);
                tma_load_2d(st + 2 * MT * 64, &mwh, c * KC, e0, &full[slot]);
                tma_load_2d(st + 2 * MT * 64 + nr * 64, &mwl, c * KC, e0, &full[slot]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t id = idesc(nr);
            for (int c = 0; c < nchunks; ++c) {
                const int slot = c % RG;
                if (!mbar_wait(&full[slot], (c / RG) & 1)) { ok = false; break; }
                tc_fence_after();
                const uint8_t* st = sm + slot * stage;
                const uint8_t *ah = st, *al = st + MT * 64, *bh = st + 2 * MT * 64, *bl = bh + nr * 64;
#pragma unroll
                for (int k = 0; k < KC / 16; ++k) {
                    const uint32_t acc = (c > 0 || k > 0) ? 1u : 0u;
                    mma_f16(tmem, umma_desc(ah, 32 * k), umma_desc(bh, 32 * k), id, acc);
                    mma_f16(tmem + nr, umma_desc(al, 32 * k), umma_desc(bh, 32 * k), id, acc);
                    mma_f16(tmem + nr, umma_desc(ah, 32 * k), umma_desc(bl, 32 * k), id, 1u);
                }
                mma_commit(&empty[slot]);
            }
            mma_commit(&done);
        }
    } else {
        if (mbar_wait(&done, 0)) {
            tc_fence_after();
            const int q = warp & 3;
            const uint32_t lane_base = (uint32_t)(q * 32) << 16;
            const int t = t0 + q * 32 + lane;
            for (int cb = 0; cb < nr; cb += 32) {
                float vh[32], vl[32];
                tmem_ld32(tmem + lane_base + cb, vh);
                tmem_ld32(tmem + lane_base + nr + cb, vl);
                if (t < T) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int e = e0 + cb + j;
                        float v = (vh[j] + vl[j]) * unscale;
                        if (bias) v += bias[e];
                        logits[(size_t)t * (E + 1) + e] = v;
                    }
                }
            }
        } else {
            ok = false;
        }
    }
    if (!ok) atomicOr(err, PI_DEVERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
}

// f16 [rows][cols] row-major, box {32 columns, box_rows rows}, SW64
bool kmajor_map(CUtensorMap* m, const __half* base, int64_t rows, int64_t cols, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(__half)};
    const cuuint32_t box[2] = {(cuuint32_t)KC, (cuuint32_t)box_rows};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}
int router_rows_per_cta(int E) { return E % 128 == 0 ? 128 : E; }

}  // namespace

int pi_prefill_prepare(pi_ctx* ctx, pi_moe_layer* L) {
    L->maps_ok = false;
    if (L->qtype != PI_QT_Q4_0 || !pi_prefill_shape_ok(L->d, L->f)) return PI_OK;
    PiPrefillMaps& M = L->maps;
    bool ok = plain_q_map(&M.q[0][0], L->gate) && plain_q_map(&M.q[0][1], L->up) && tiled_q_map(&M.q[0][2], L->down) &&
              scale_map(&M.d[0][0], L->gate) && scale_map(&M.d[0][1], L->up) && scale_map(&M.d[0][2], L->down);
    if (ok && L->has_shared)
        ok = plain_q_map(&M.q[1][0], L->gate_sh) && plain_q_map(&M.q[1][1], L->up_sh) &&
             tiled_q_map(&M.q[1][2], L->down_sh) && scale_map(&M.d[1][0], L->gate_sh) &&
             scale_map(&M.d[1][1], L->up_sh) && scale_map(&M.d[1][2], L->down_sh);
    if (!ok) return pi_set_error(ctx, PI_ERR_CUDA, "prefill GEMM: cuTensorMapEncodeTiled failed for the weights");
    L->maps_ok = true;
    return PI_OK;
}

int pi_prefill_experts(pi_ctx* ctx, const pi_moe_layer* L, const ExpertArgs& a, int64_t max_items, int64_t n_slots,
                       const __half* xth, const __half* xtl, int64_t T, __half* hh, __half* hl, cudaStream_t st) {
    if (L->qtype != PI_QT_Q4_0) return pi_set_error(ctx, PI_ERR_ARG, "prefill GEMM: Q4_0 weights only");
    static_assert(MT * DN_MPC == 512 && MT * GU_MPC == 128, "pi_prefill_shape_ok matches the CTA blocks");
    if (!pi_prefill_shape_ok(a.d, a.f) || (L->has_shared && L->f_sh != L->f))
        return pi_set_error(ctx, PI_ERR_ARG,
                            "prefill GEMM: n_embd must be a multiple of 512, expert widths equal and a multiple of 128");
    if (!L->maps_ok) return pi_set_error(ctx, PI_ERR_CUDA, "prefill GEMM: weight tensor maps unavailable");
    CUtensorMap mhh, mhl;
    if (!act_map(&mhh, hh, n_slots, a.f) || !act_map(&mhl, hl, n_slots, a.f))
        return pi_set_error(ctx, PI_ERR_CUDA, "prefill GEMM: cuTensorMapEncodeTiled failed");
    pi_smem_attr((const void*)k_moe_gemm<0>, gemm_smem<0>());
    pi_smem_attr((const void*)k_moe_gemm<1>, gemm_smem<1>());
    {
        PiProfScope ps(ctx, st, "k_gemm_gateup");
        k_moe_gemm<0><<<dim3((unsigned)(a.f / (MT * GU_MPC)), (unsigned)max_items), GT, gemm_smem<0>(), st>>>(
            a, L->maps, mhh, mhl, xth, xtl, hh, hl, ctx->dev_err);
    }
    {
        PiProfScope ps(ctx, st, "k_gemm_down");
        k_moe_gemm<1><<<dim3((unsigned)(a.d / (MT * DN_MPC)), (unsigned)max_items), GT, gemm_smem<1>(), st>>>(
            a, L->maps, mhh, mhl, xth, xtl, hh, hl, ctx->dev_err);
    }
    return pi_cuda_check(ctx, cudaGetLastError(), "prefill GEMM") ? PI_ERR_CUDA : PI_OK;
}

bool pi_router_maps(pi_moe_layer* L) {
    const int nr = router_rows_per_cta(L->E);
    return kmajor_map(&L->rmap_h, L->router_h, L->E, L->d, nr) && kmajor_map(&L->rmap_l, L->router_l, L->E, L->d, nr);
}

int pi_router_logits_tc(pi_ctx* ctx, const pi_moe_layer* L, const __half* xh, const __half* xl, int64_t T,
                        float* logits, cudaStream_t st) {
    const int nr = router_rows_per_cta(L->E);
    CUtensorMap mxh, mxl;
    if (!kmajor_map(&mxh, xh, T, L->d, MT) || !kmajor_map(&mxl, xl, T, L->d, MT))
        return pi_set_error(ctx, PI_ERR_CUDA, "router: cuTensorMapEncodeTiled failed");
    const size_t smem = (size_t)RG * 2 * (MT + nr) * 64 + 1024;
    pi_smem_attr((const void*)k_router_gemm, RG * 2 * (MT + 256) * 64 + 1024);
    PiProfScope ps(ctx, st, "k_router_gemm");
    k_router_gemm<<<dim3((unsigned)((T + MT - 1) / MT), (unsigned)(L->E / nr)), 192, smem, st>>>(
        mxh, mxl, L->rmap_h, L->rmap_l, (int)T, (int)L->d, L->E, nr, ldexpf(1.0f, -L->router_rs), L->bias, logits,
        ctx->dev_err);
    return pi_cuda_check(ctx, cudaGetLastError(), "router GEMM") ? PI_ERR_CUDA : PI_OK;
}
