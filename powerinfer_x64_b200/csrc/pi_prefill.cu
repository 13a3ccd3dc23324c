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
// Work item: (expert e, tile of 128 weight rows, <= 128 slots of e). The CTA
// (256 threads) walks K in 64-element chunks with two shared-memory stages:
//   * every thread dequantises half a weight row of the chunk (one Q4_0
//     block: nibbles in reference order times the f16 block scale) into hi/lo
//     f16 tiles and copies one slot row of the hi or lo activations, both in
//     the canonical K-major 128-byte-swizzled layout of the UMMA descriptors,
//     from registers loaded one chunk ahead;
//   * thread 0 issues the MMAs and a tcgen05.commit onto the stage's mbarrier,
//     which tells the loaders when the stage may be overwritten.
// The epilogue reads the accumulators with tcgen05.ld (warp w owns TMEM lanes
// 32w..32w+31, one weight row per thread) and writes SwiGLU h (gate/up) or y
// (down). All mbarrier waits are bounded (1 s) and report PI_DEVERR_TIMEOUT.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "pi_common.cuh"
#include "pi_internal.h"

namespace {

constexpr int NT = PI_GEMM_NT;  // slots per item (MMA N)
constexpr int MT = 128;         // weight rows per item (MMA M)
constexpr int KC = 64;          // K elements per chunk (one 128-byte swizzle atom)
constexpr int TILE_BYTES = 128 * 128;  // 128 rows x 128 bytes

PI_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

PI_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
PI_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// true once the phase with this parity completed; false after ~1 s
PI_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 255) == 0) {
            const uint64_t now = globaltimer_ns();
            if (i == 0) t0 = now;
            else if (now - t0 > 1000000000ull) return false;
        }
    }
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes (SBO = 1024), version 1 (sm_100).
PI_DEV uint64_t umma_desc(const void* tile, uint32_t byte_offset) {
    const uint32_t a = smem_u32(tile) + byte_offset;
    uint64_t d = (uint64_t)((a >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;            // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;  // SBO
    d |= (uint64_t)1 << 46;            // version
    d |= (uint64_t)2 << 61;            // SWIZZLE_128B
    return d;
}
// instruction descriptor: f16 x f16 -> f32, both K-major, M = 128, N = NT
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(MT >> 4) << 24);

PI_DEV void mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(IDESC), "r"(accumulate)
        : "memory");
}
PI_DEV void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
PI_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
PI_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PI_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
PI_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// 2-D tiled TMA load (no multicast) of box {64 f16, 128 rows} at element (x, y)
PI_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
PI_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive f32 accumulator columns of this thread's TMEM lane
PI_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// swizzled position of 16-byte chunk c (0..7) of row r in a K-major SW128 tile
PI_DEV int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// half a row (one 32-element block, h = 0/1) x 64 K -> 4 swizzled chunks each of hi/lo.
// Packed f16 arithmetic: 0x6400 | n is the f16 value 1024 + n, so (0x6400 | n) - 1032 = n - 8
// exactly; hi = rn(d * (n - 8)) is one rounding of the exact product, the same value as
// rounding the f32 product (exact: 11 x 4 bits); lo = rn(d * (n - 8) - hi) by one fused
// multiply-add, the same value as rounding the exact f32 difference.
PI_DEV void dequant_half_q4(const int4 nib, __half sc, uint8_t* th, uint8_t* tl, int r, int h) {
    const uint32_t w[4] = {(uint32_t)nib.x, (uint32_t)nib.y, (uint32_t)nib.z, (uint32_t)nib.w};
    const __half2 d2 = __half2half2(sc);
    const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6408));  // 1032
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
        const int c = 4 * h + cc;
        const uint32_t v = w[cc];
        // t_j holds nibble j (bits 0..3) and nibble j + 4 (bits 16..19): elements j, j + 4
        uint32_t t[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) t[j] = (v >> (4 * j)) & 0x000F000Fu;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            // pair p = elements (2p, 2p + 1): low halves of t[2p], t[2p+1] for p < 2, high halves after
            const uint32_t a = t[(2 * p) & 3], b = t[(2 * p + 1) & 3];
            const uint32_t q = (p < 2 ? __byte_perm(a, b, 0x5410) : __byte_perm(a, b, 0x7632)) | 0x64006400u;
            const __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&q), off);
            const __half2 hv = __hmul2(d2, qv);
            const __half2 lv = __hfma2(d2, qv, __hneg2(hv));
            hi[p] = *reinterpret_cast<const uint32_t*>(&hv);
            lo[p] = *reinterpret_cast<const uint32_t*>(&lv);
        }
        *reinterpret_cast<uint4*>(th + swz(r, c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(tl + swz(r, c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// Q4_0 weight row r of a plain SoA matrix (nibbles [rows][K/2], scales [rows][K/32])
struct Q4Plain {
    const uint8_t* q;
    const __half* d;
    int K;
    // block 2c + h of row r: 16 nibble bytes and its scale
    PI_DEV void load_half(int r, int c, int h, int4& n, __half& sc) const {
        n = *reinterpret_cast<const int4*>(q + (size_t)r * (K / 2) + c * 32 + 16 * h);
        sc = d[(size_t)r * (K / 32) + 2 * c + h];
    }
};
// Q4_0 down projection in the decode kernels' lane-tiled order (pi_tile_down_mats):
// 16-byte chunk j of row r lives at (r/8)*8*nch + ((j % cpq)*32 + 4*(r%8) + j/cpq)*16.
struct Q4Tiled {
    const uint8_t* q;
    const __half* d;
    int K;
    PI_DEV const uint8_t* chunk(int r, int j) const {
        const int nch = K / 32, cpq = nch / 4;
        return q + ((size_t)(r >> 3) * 8 * nch + (size_t)(j % cpq) * 32 + (r & 7) * 4 + j / cpq) * 16;
    }
    PI_DEV void load_half(int r, int c, int h, int4& n, __half& sc) const {
        n = *reinterpret_cast<const int4*>(chunk(r, 2 * c + h));
        sc = d[(size_t)r * (K / 32) + 2 * c + h];
    }
};

// MODE 0: gate/up (two accumulators, 256 TMEM columns); MODE 1: down (one).
// Warp roles:
//   0-7  converters: dequantise each 64-K weight chunk into one of two weight
//        stages (thread t: row t / 2, block 2c + t % 2, loaded one chunk ahead
//        into registers), then arrive on the stage's `full` barrier; after the
//        last chunk of an m-tile they run its epilogue;
//   8    TMA producer: streams the activation chunks (f16 hi and lo, already in
//        slot order) into a three-deep ring;
//   9    MMA issuer: waits for a weight stage and its activation slot, issues
//        the MMAs and releases both with tcgen05.commit.
constexpr int GT = 320;
constexpr int XS = 3;  // activation ring depth
constexpr int GU_MPC = 1, DN_MPC = 4;  // 128-row m-tiles handled by one CTA (gate/up, down)
template <int MODE>
__global__ __launch_bounds__(GT, 1) void k_moe_gemm(ExpertArgs a, const __grid_constant__ CUtensorMap map_hi,
                                                    const __grid_constant__ CUtensorMap map_lo,
                                                    __half* __restrict__ hh, __half* __restrict__ hl, uint32_t* err) {
    constexpr int NMAT = MODE == 0 ? 2 : 1;         // weight matrices per item
    constexpr int WSTAGE = 2 * NMAT * TILE_BYTES;   // W hi/lo per matrix
    constexpr uint32_t TCOLS = MODE == 0 ? 256 : 128;
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* xring = sm + 2 * WSTAGE;  // XS slots of {hi, lo} tiles
    __shared__ __align__(8) uint64_t wbar[2], full[2], xfull[XS], xempty[XS];
    __shared__ uint32_t s_tmem;
    const int tid = threadIdx.x, warp = tid >> 5;
    const int it = blockIdx.y;
    if (it >= *a.n_items) return;
    const int4 item = a.items[it];
    const bool sh = item.x == a.E;
    constexpr int mpc = MODE == 0 ? GU_MPC : DN_MPC;  // m-tiles per CTA
    const int row0 = blockIdx.x * mpc * MT;
    const int K = MODE == 0 ? a.d : a.f;
    const int nchunks = K / KC;
    const int n_iter = mpc * nchunks;

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&wbar[i], 1);
            mbar_init(&full[i], 8);  // one arrival per converter warp
        }
        for (int i = 0; i < XS; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], 1);
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
        // activation producer: chunk g -> ring slot g % XS once the MMAs of chunk g - XS are done
        if ((tid & 31) == 0) {
            for (int g = 0; g < n_iter; ++g) {
                const int slot = g % XS, use = g / XS;
                if (use > 0 && !mbar_wait(&xempty[slot], (use - 1) & 1)) { ok = false; break; }
                uint8_t* xt = xring + slot * 2 * TILE_BYTES;
                mbar_expect_tx(&xfull[slot], 2 * TILE_BYTES);
                const int xc = (g % nchunks) * KC;
                tma_load_2d(xt, &map_hi, xc, item.y, &xfull[slot]);
                tma_load_2d(xt + TILE_BYTES, &map_lo, xc, item.y, &xfull[slot]);
            }
        }
    } else if (warp == 9) {
        if ((tid & 31) == 0) {
            for (int g = 0; g < n_iter; ++g) {
                const int s = g & 1, slot = g % XS, c = g % nchunks;
                if (!mbar_wait(&full[s], (g >> 1) & 1) || !mbar_wait(&xfull[slot], (g / XS) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint8_t* st = sm + s * WSTAGE;
                const uint8_t* xt = xring + slot * 2 * TILE_BYTES;
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const uint8_t* wh = st + 2 * m * TILE_BYTES;
                    const uint8_t* wl = wh + TILE_BYTES;
                    const uint32_t dcol = tmem + m * NT;
#pragma unroll
                    for (int k = 0; k < KC / 16; ++k) {
                        const uint64_t dwh = umma_desc(wh, 32 * k), dwl = umma_desc(wl, 32 * k);
                        const uint64_t dxh = umma_desc(xt, 32 * k), dxl = umma_desc(xt + TILE_BYTES, 32 * k);
                        mma_f16(dcol, dwh, dxh, (c > 0 || k > 0) ? 1u : 0u);
                        mma_f16(dcol, dwl, dxh, 1u);
                        mma_f16(dcol, dwh, dxl, 1u);
                    }
                }
                mma_commit(&wbar[s]);
                mma_commit(&xempty[slot]);
            }
        }
    } else {
        const size_t mat = sh ? 0 : (size_t)item.x * (MODE == 0 ? a.f : a.d);
        Q4Plain wg{}, wu{};
        Q4Tiled wd{};
        if (MODE == 0) {
            wg = Q4Plain{(const uint8_t*)(sh ? a.gs : a.g) + mat * (a.d / 2), (sh ? a.gsd : a.gd) + mat * (a.d / 32), a.d};
            wu = Q4Plain{(const uint8_t*)(sh ? a.us : a.u) + mat * (a.d / 2), (sh ? a.usd : a.ud) + mat * (a.d / 32), a.d};
        } else {
            wd = Q4Tiled{(const uint8_t*)(sh ? a.dns : a.dn) + mat * (a.f / 2), (sh ? a.dsd : a.dd) + mat * (a.f / 32),
                         a.f};
        }
        // thread t dequantises row t / 2, block (2c + t % 2) of each chunk c: a warp reads whole sectors
        const int rw = tid >> 1, hw = tid & 1;
        int4 pn[NMAT];
        __half ps[NMAT];
        auto prefetch = [&](int g) {
            const int wr = row0 + (g / nchunks) * MT + rw, c = g % nchunks;
            if (MODE == 0) {
                wg.load_half(wr, c, hw, pn[0], ps[0]);
                wu.load_half(wr, c, hw, pn[NMAT - 1], ps[NMAT - 1]);
            } else {
                wd.load_half(wr, c, hw, pn[0], ps[0]);
            }
        };
        prefetch(0);
        for (int g = 0; g < n_iter; ++g) {
            const int s = g & 1, mi = g / nchunks, c = g % nchunks;
            int4 cn[NMAT];
            __half cs[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) { cn[m] = pn[m]; cs[m] = ps[m]; }
            if (g + 1 < n_iter) prefetch(g + 1);
            if (g >= 2 && !mbar_wait(&wbar[s], ((g - 2) >> 1) & 1)) { ok = false; break; }
            uint8_t* st = sm + s * WSTAGE;
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
                dequant_half_q4(cn[m], cs[m], st + 2 * m * TILE_BYTES, st + (2 * m + 1) * TILE_BYTES, rw, hw);
            fence_async_smem();
            tc_fence_before();  // orders this warp's earlier TMEM reads (epilogue) before the next MMAs
            __syncwarp();
            if ((tid & 31) == 0) mbar_arrive(&full[s]);
            if (c + 1 < nchunks) continue;
            // last chunk of m-tile mi: wait for its MMAs, then the epilogue. The next
            // m-tile's first MMA (issued once every converter warp has arrived on the next
            // stage, i.e. after this epilogue) overwrites TMEM.
            if (!mbar_wait(&wbar[s], (g >> 1) & 1)) { ok = false; break; }
            tc_fence_after();
            // TMEM lane (warp % 4) * 32 + lane = weight row; warps 0-3 take slot
            // columns [0, 64), warps 4-7 [64, 128)
            const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
            const int row = row0 + mi * MT + (warp & 3) * 32 + (tid & 31);
            const int c0 = (warp >> 2) * (NT / 2);
            for (int cb = c0; cb < c0 + NT / 2; cb += 32) {
                if (cb >= item.z) break;
                float gv[32];
                tmem_ld32(tmem + lane_base + cb, gv);
                if (MODE == 0) {
                    float u[32];
                    tmem_ld32(tmem + lane_base + NT + cb, u);
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

// xh/xl[slot] = f16 hi/lo split of the f32 token row of slot (routed slots via
// perm, then one slot per token for the shared expert); 8 elements per thread
__global__ void k_split_slots(const float* __restrict__ x, const int32_t* __restrict__ perm, int n_routed,
                              int64_t n_slots, int d, __half* __restrict__ xh, __half* __restrict__ xl) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int per = d / 8;
    if (i >= n_slots * per) return;
    const int64_t slot = i / per;
    const int c = (int)(i % per) * 8;
    const int64_t tok = slot < n_routed ? perm[slot] : slot - n_routed;
    const float4 v0 = *reinterpret_cast<const float4*>(x + tok * d + c);
    const float4 v1 = *reinterpret_cast<const float4*>(x + tok * d + c + 4);
    const float f[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const __half2 hv = __floats2half2_rn(f[2 * p], f[2 * p + 1]);
        const float2 hf = __half22float2(hv);
        const __half2 lv = __floats2half2_rn(f[2 * p] - hf.x, f[2 * p + 1] - hf.y);
        hi[p] = *reinterpret_cast<const uint32_t*>(&hv);
        lo[p] = *reinterpret_cast<const uint32_t*>(&lv);
    }
    *reinterpret_cast<uint4*>(xh + slot * d + c) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(xl + slot * d + c) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

template <int MODE>
constexpr size_t gemm_smem() {
    return (size_t)(2 * (MODE == 0 ? 4 : 2) + 2 * XS) * TILE_BYTES + 1024;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// f16 [rows][cols] row-major, box {64 columns, 128 rows}, 128-byte swizzle
// (the UMMA K-major SW128 layout); rows past the end read as zeros
bool make_map(CUtensorMap* m, const __half* base, int64_t rows, int64_t cols) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * sizeof(__half)};
    const cuuint32_t box[2] = {(cuuint32_t)KC, 128};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int pi_prefill_experts(pi_ctx* ctx, const ExpertArgs& a, int qtype, int64_t max_items, int64_t n_slots, __half* xh,
                       __half* xl, __half* hh, __half* hl, cudaStream_t st) {
    if (qtype != PI_QT_Q4_0) return pi_set_error(ctx, PI_ERR_ARG, "prefill GEMM: Q4_0 weights only");
    static_assert(MT * DN_MPC == 512 && MT * GU_MPC == 128, "pi_prefill_shape_ok matches the CTA blocks");
    if (!pi_prefill_shape_ok(a.d, a.f))
        return pi_set_error(ctx, PI_ERR_ARG, "prefill GEMM: n_embd must be a multiple of 512, expert width of 128");
    CUtensorMap mxh, mxl, mhh, mhl;
    if (!make_map(&mxh, xh, n_slots, a.d) || !make_map(&mxl, xl, n_slots, a.d) || !make_map(&mhh, hh, n_slots, a.f) ||
        !make_map(&mhl, hl, n_slots, a.f))
        return pi_set_error(ctx, PI_ERR_CUDA, "prefill GEMM: cuTensorMapEncodeTiled failed");
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_moe_gemm<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<0>());
        cudaFuncSetAttribute(k_moe_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<1>());
        attr = true;
    }
    {
        PiProfScope ps(ctx, st, "k_split_slots");
        const int64_t n = n_slots * (a.d / 8);
        k_split_slots<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a.xf, a.perm, a.n_routed, n_slots, a.d, xh, xl);
    }
    {
        PiProfScope ps(ctx, st, "k_gemm_gateup");
        k_moe_gemm<0><<<dim3((unsigned)(a.f / (MT * GU_MPC)), (unsigned)max_items), GT, gemm_smem<0>(), st>>>(
            a, mxh, mxl, hh, hl, ctx->dev_err);
    }
    {
        PiProfScope ps(ctx, st, "k_gemm_down");
        k_moe_gemm<1><<<dim3((unsigned)(a.d / (MT * DN_MPC)), (unsigned)max_items), GT, gemm_smem<1>(), st>>>(
            a, mhh, mhl, hh, hl, ctx->dev_err);
    }
    return pi_cuda_check(ctx, cudaGetLastError(), "prefill GEMM") ? PI_ERR_CUDA : PI_OK;
}
