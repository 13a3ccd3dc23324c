// Prefill-sized Q8_0 expert products (Q8_0, T = 8192) on the
// tensor cores, bit-exact with the reference.
//
// The reference's Q8_0 matvec (quant/mod.rs:939-957) quantises the activations
// to Q8_0 and sums, block by block in ascending order,
//     acc += (float)sumi_b * (d_w,b * d_x,b),   sumi_b = sum_{k in b} q_w q_x,
// in f32 starting from 0. Here the int8 values of both operands are held as
// exact f16 and multiplied with tcgen05.mma kind::f16: every product and every
// partial sum of a block is an integer below 2^20, so the f32 result in TMEM is
// exactly (float)sumi_b. The scale product d_w,b * d_x,b of every (slot, row) is
// made on the tensor cores too: both scales are f16 values, so their product
// (22 significant bits) is exact in f32, and one K = 16 MMA of a slot-scale column
// by a row-scale row writes all of them. Per block a fresh pair of accumulators
// (sumi, scale product) lands in TMEM and epilogue warps add sumi * product to
// f32 registers in block order (one multiply, one add per output and block), so
// each output is the reference's own sequence of roundings. The gate/up kernel
// applies the reference's SwiGLU and quantises h to Q8_0 per 32 rows, exactly as
// ffn_swiglu_q does before its down matvec (quant/mod.rs:1184-1249); the down
// kernel writes y.
//
// Orientation: the token rows of a work item (<= 128 slots) are the MMA's M
// side and 128 weight rows its N side, so a TMEM lane is one slot, a thread of
// the epilogue owns one slot, and a 32-row Q8_0 block of h lies in one thread's
// registers.
//
// Operands:
//   A (slots)   gate/up: each converter thread gathers its slot's token row of the
//               quantised activations (int8, through the dispatch permutation; the
//               next stage's words are requested while this one is converted) and
//               writes exact f16 into the 64-byte-swizzled tile the MMA reads;
//               down: h as f16 rows [slots][f] in slot order (the gate/up epilogue
//               writes them so), loaded by TMA with the same swizzle;
//   B (weights) int8 rows of the lane-tiled decode layouts, loaded raw by TMA in
//               groups of 4 blocks and turned into exact f16 by converter warps;
//   scales      per block a [128 x 16] f16 tile of slot scales (column 0) and one
//               of row scales (column 0), written by the converters (no swizzle).
//
// The kernel is persistent: a CTA walks tiles (work item, 128 weight rows) and
// its pipeline runs on across tile boundaries. Warp roles (QT = 448 threads):
//   0-7   epilogue: warp w owns slots 32 (w % 4) .. +31 (TMEM lanes) and, for
//         gate/up, gate columns 32 (w / 4) .. +31 with their up columns (+64),
//         for down, columns 64 (w / 4) .. +63;
//   8-11  converters: thread c converts weight row c of each block, for gate/up
//         also slot c's activation row, and writes the scale tiles' row c (its
//         row's scale, slot c's scale);
//   12    MMA issuer;  13 TMA producer.
// Every mbarrier wait is bounded and reports PI_DEVERR_TIMEOUT.
#include "pi_tc.cuh"
// pi_tc.cuh (pi_common.cuh) comes first: it names the quant types that pi_moe.h defines as macros
#include "pi_internal.h"

namespace {
using namespace pitc;

constexpr int QN = PI_GEMM_NT_Q8;  // slots per work item (MMA M)
constexpr int TN = 128;            // weight rows per tile (MMA N)
constexpr int NEPI = 8, NCONV = 4;
constexpr int QT = (NEPI + NCONV + 2) * 32;
constexpr int G4 = 4;              // blocks per raw weight group
constexpr int RG = 2;              // raw weight groups in flight
constexpr int PB = 2;              // blocks per operand stage (one handshake)
constexpr int TS = 4;              // operand stages of PB blocks
constexpr int DB = 2;              // TMEM buffers of one block: sumi (TN columns) + scale product (TN)
constexpr int TILE = 128 * 64;     // 128 rows x 32 f16, 64-byte swizzle
constexpr int STILE = 128 * 32;    // 128 rows x 16 f16, no swizzle (scale tiles)
constexpr int STAGE = PB * (2 * TILE + 2 * STILE);  // per block {A, B, slot scales, row scales}
constexpr int RAWW = TN * G4 * 32;    // weight rows of a group (16 KB)
static_assert(G4 == 2 * PB, "a raw group fills two stages");
static_assert(QN == 128, "the MMA M side is 128 slots");
static_assert(DB * 2 * TN == 512, "the TMEM buffers fill the 512 columns");
constexpr size_t QSMEM = (size_t)TS * STAGE + (size_t)RG * RAWW + 1024;

// UMMA shared-memory descriptor of a K-major tile without swizzle: core matrices of
// 8 rows x 16 bytes; K-adjacent cores LBO = 128 bytes apart, 8-row groups SBO = 256.
PI_DEV uint64_t umma_desc_plain(const void* tile) {
    const uint32_t a = smem_u32(tile);
    uint64_t d = (uint64_t)((a >> 4) & 0x3FFF);
    d |= (uint64_t)(128 >> 4) << 16;  // LBO
    d |= (uint64_t)(256 >> 4) << 32;  // SBO
    d |= (uint64_t)1 << 46;           // version; layout type 0 = no swizzle
    return d;
}
// byte offset of row r, K elements 0..7 in a plain [128 x 16] scale tile
PI_DEV int stile_row(int r) { return (r >> 3) * 256 + (r & 7) * 16; }

// 16 int8 (one 16-byte word) -> 16 exact f16, the 16-byte chunks c0 and c0 + 1 of
// swizzled row r of a SW64 tile: 0x6400 | (b ^ 0x80) is the f16 value 1024 + b + 128,
// so subtracting 1152 gives b.
PI_DEV void int8x16_to_f16(const uint4 a, uint8_t* tile, int r, int c0) {
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
    const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152
#pragma unroll
    for (int c = 0; c < 2; ++c) {  // chunk c0 + c = elements 8c .. 8c+7 of the word
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
        *reinterpret_cast<uint4*>(tile + swz(r, c0 + c)) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// The Q8_0 activation quantiser (quant/mod.rs:698-736) on 32 values held by one
// thread: amax -> d = amax/127 -> id = 1/d -> q = clamp(round(x*id)); the stored
// scale is f16(d). Same arithmetic as warp_quant_q8, without the shuffles.
PI_DEV float quant_block32(const float (&x)[32], int8_t (&q)[32]) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float a = fabsf(x[i]);
        amax = (a == a) ? fmaxf(amax, a) : amax;
    }
    const float d = fdiv(amax, 127.0f);
    const float id = (d != 0.0f) ? fdiv(1.0f, d) : 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float r = roundf(fmul(x[i], id));
        q[i] = (int8_t)((r != r) ? 0 : (int)fminf(127.0f, fmaxf(-127.0f, r)));
    }
    return __half2float(__float2half_rn(d));
}

struct TileRef {
    int4 item;
    int mt;
};

// MODE 0: gate/up (+ SwiGLU, Q8_0 h as exact f16); MODE 1: down (y).
template <int MODE, bool FAST>
__global__ __launch_bounds__(QT, 1) void k_moe_gemm_q8(ExpertArgs a, const __grid_constant__ PiPrefillMaps wm,
                                                       const __grid_constant__ CUtensorMap mact,
                                                       const float* __restrict__ xsc, int64_t n_slots, uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* tiles = sm;              // TS stages of PB x {A tile, B tile, slot-scale tile, row-scale tile}
    uint8_t* raws = sm + TS * STAGE;  // RG raw weight groups
    __shared__ __align__(8) uint64_t tile_full[TS], tile_free[TS], d_full[DB], d_free[DB];
    __shared__ __align__(8) uint64_t raw_full[RG], raw_free[RG];
    __shared__ uint32_t s_tmem;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = MODE == 0 ? a.d : a.f;
    const int n_routed = a.n_routed_dev ? *a.n_routed_dev : a.n_routed;  // routed slots (gate/up gathers)
    const int nb = K / 32, ng = nb / G4;
    const int MT = MODE == 0 ? a.f / 64 : a.d / TN;  // weight-row tiles per item
    const int n_tiles = *a.n_items * MT;
    if ((int)blockIdx.x >= n_tiles) return;
    auto tile_at = [&](int t) {
        TileRef r;
        r.item = a.items[t / MT];
        r.mt = t % MT;
        return r;
    };
    auto a_tile = [&](int ts, int b) { return tiles + ts * STAGE + b * (2 * TILE + 2 * STILE); };

    if (tid == 0) {
        for (int i = 0; i < TS; ++i) {
            mbar_init(&tile_full[i], MODE == 0 ? NCONV : NCONV + 1);  // gate/up: the converters write A too
            mbar_init(&tile_free[i], 1);
        }
        for (int i = 0; i < DB; ++i) {
            mbar_init(&d_full[i], 1);
            mbar_init(&d_free[i], NEPI);
        }
        for (int i = 0; i < RG; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_free[i], NCONV);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // the scale tiles are zero but for column 0, which the converters rewrite per block
    for (int ts = 0; ts < TS; ++ts)
        for (int b = 0; b < PB; ++b)
            for (int i = tid; i < 2 * STILE / 16; i += QT)
                reinterpret_cast<uint4*>(a_tile(ts, b) + 2 * TILE)[i] = make_uint4(0, 0, 0, 0);
    fence_async_smem();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(DB * 2 * TN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ok = true;

    if (warp == NEPI + NCONV + 1) {
        // ---- TMA producer: raw weight groups and activation tiles ----
        int g = 0;
        for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
            const TileRef tr = tile_at(t);
            const bool sh = tr.item.x == a.E;
            const int mrow = (sh ? 0 : tr.item.x * (MODE == 0 ? a.f : a.d));
            for (int q = 0; q < ng; ++q, ++g) {
                const int slot = g % RG;
                int w_ok = 1;
                if (lane == 0) {
                    if (g >= RG && !mbar_wait(&raw_free[slot], (g / RG - 1) & 1)) w_ok = 0;
                    else {
                        mbar_expect_tx(&raw_full[slot], RAWW);
                        uint8_t* rw = raws + slot * RAWW;
                        if (MODE == 0) {
                            // lane-tiled gate/up rows: half h of block B at ((B/32)*64 + h*32 + B%32) * 16
                            // bytes, so the first halves of blocks 4q..4q+3 are 64 contiguous bytes, the
                            // second ones +512
                            const int b0 = G4 * q, x0 = ((b0 >> 5) * 64 + (b0 & 31)) * 16;
                            const int r0 = mrow + tr.mt * 64;
                            const CUtensorMap* mg = sh ? &wm.q[1][0] : &wm.q[0][0];
                            const CUtensorMap* mu = sh ? &wm.q[1][1] : &wm.q[0][1];
                            tma_load_2d(rw, mg, x0, r0, &raw_full[slot]);
                            tma_load_2d(rw + 64 * 64, mg, x0 + 512, r0, &raw_full[slot]);
                            tma_load_2d(rw + 2 * 64 * 64, mu, x0, r0, &raw_full[slot]);
                            tma_load_2d(rw + 3 * 64 * 64, mu, x0 + 512, r0, &raw_full[slot]);
                        } else {
                            // lane-tiled down rows: chunk j of row r at ((r/8)*8*nch + (j%cpq)*32 + (r%8)*4
                            // + j/cpq) * 16, blocks 4q..4q+3 = chunks 8q..8q+7 = all j%cpq with j/cpq = q
                            const CUtensorMap* md = sh ? &wm.q[1][2] : &wm.q[0][2];
                            tma_load_4d(rw, md, q * 16, 0, 0, (mrow + tr.mt * TN) >> 3, &raw_full[slot]);
                        }
                    }
                    for (int pi = 0; pi < G4 / PB && w_ok && MODE == 1; ++pi) {
                        const int s = (G4 / PB) * g + pi, ts = s % TS;
                        if (s >= TS && !mbar_wait(&tile_free[ts], (s / TS - 1) & 1)) { w_ok = 0; break; }
                        mbar_expect_tx(&tile_full[ts], PB * TILE);
                        for (int b = 0; b < PB; ++b)
                            tma_load_2d(a_tile(ts, b), &mact, (G4 * q + PB * pi + b) * 32, tr.item.y, &tile_full[ts]);
                    }
                }
                if (!__shfl_sync(0xffffffffu, w_ok, 0)) { ok = false; break; }
            }
        }
        // let the last copies land before the CTA can exit (bounded; only matters after a timeout)
        if (lane == 0 && g > 0) mbar_wait(&raw_full[(g - 1) % RG], ((g - 1) / RG) & 1);
    } else if (warp >= NEPI && warp < NEPI + NCONV) {
        // ---- converters: thread c converts weight row c and writes row c of both scale tiles ----
        const int row = tid - NEPI * 32;
        int g = 0;
        for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
            const TileRef tr = tile_at(t);
            const bool sh = tr.item.x == a.E;
            const int mrow = (sh ? 0 : tr.item.x * (MODE == 0 ? a.f : a.d));
            const __half* wd;
            int wr;
            if (MODE == 0) {
                const bool up = row >= 64;
                wd = up ? (sh ? a.usd : a.ud) : (sh ? a.gsd : a.gd);
                wr = mrow + tr.mt * 64 + (row & 63);
            } else {
                wd = sh ? a.dsd : a.dd;
                wr = mrow + tr.mt * TN + row;
            }
            const __half* scp = wd + (size_t)wr * nb;
            const int64_t srow = (int64_t)tr.item.y + row;  // this thread's slot (scale row of the A side)
            const float* xsp = srow < n_slots ? xsc + srow * nb : nullptr;
            // gate/up: the slot's token row (int8) and scales, gathered here (routed slot s
            // reads token perm[s], shared slot n_routed + t reads row sh_row0 + t)
            const int8_t* xrow = nullptr;
            if (MODE == 0) {
                xsp = nullptr;
                if (row < tr.item.z) {
                    const bool shs = srow >= n_routed;
                    const int64_t tok = shs ? a.sh_row0 + (srow - n_routed) : a.perm[srow];
                    xrow = (shs && a.xq_sh ? a.xq_sh : a.xq) + tok * K;
                    xsp = (shs && a.xs_sh ? a.xs_sh : a.xs) + tok * nb;
                }
            }
            // the row's weight scales and the slot's activation scales of group q, as f16 bits
            auto load_sc = [&](int q, uint2& w, uint2& x) {
                w = *reinterpret_cast<const uint2*>(scp + G4 * q);
                x = make_uint2(0, 0);
                if (xsp) {  // activation scales are f16 values held in f32: exact conversions
                    const float4 f = *reinterpret_cast<const float4*>(xsp + G4 * q);
                    const __half2 lo = __floats2half2_rn(f.x, f.y), hi = __floats2half2_rn(f.z, f.w);
                    x = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
                }
            };
            // raw position of this row's 16-byte half h of block i
            auto raw_half = [&](const uint8_t* rg, int i, int h) -> const uint8_t* {
                if (MODE == 0) return rg + (row >> 6) * 2 * 64 * 64 + h * 64 * 64 + (row & 63) * 64 + 16 * i;
                return rg + (row >> 3) * 1024 + (2 * i + h) * 128 + (row & 7) * 16;  // [r/8][chunk][r%8][16 B]
            };
            // Chunk j (0..3) of this row's stage pi -> (block i, half h); gate/up rows are 64 bytes
            // apart, so the block is rotated per row pair to spread a load over the banks
            auto chunk_of = [&](int pi, int j, int& i, int& h) {
                if (MODE == 0) {
                    i = PB * pi + ((j + (row >> 1)) & 1);
                    h = j >> 1;
                } else {
                    i = PB * pi + (j >> 1);
                    h = j & 1;
                }
            };
            uint2 w_cur, x_cur, w_nxt, x_nxt;
            load_sc(0, w_cur, x_cur);
            uint4 an[2 * PB];  // gate/up: the next stage's activation words (int8 zeros past the slot count)
#pragma unroll
            for (int j = 0; j < 2 * PB; ++j)
                an[j] = MODE == 0 && xrow ? *reinterpret_cast<const uint4*>(xrow + 16 * j) : make_uint4(0u, 0u, 0u, 0u);
            for (int q = 0; q < ng; ++q, ++g) {
                const int slot = g % RG;
                if (q + 1 < ng) load_sc(q + 1, w_nxt, x_nxt);
                if (!mbar_wait(&raw_full[slot], (g / RG) & 1)) { ok = false; break; }
                const uint8_t* rg = raws + slot * RAWW;
                const uint16_t wv[4] = {(uint16_t)(w_cur.x & 0xffff), (uint16_t)(w_cur.x >> 16),
                                        (uint16_t)(w_cur.y & 0xffff), (uint16_t)(w_cur.y >> 16)};
                const uint16_t xv[4] = {(uint16_t)(x_cur.x & 0xffff), (uint16_t)(x_cur.x >> 16),
                                        (uint16_t)(x_cur.y & 0xffff), (uint16_t)(x_cur.y >> 16)};
#pragma unroll
                for (int pi = 0; pi < G4 / PB; ++pi) {  // one stage (PB blocks) at a time
                    const int s = (G4 / PB) * g + pi;
                    // gate/up: this stage's activations are in av; request the next stage's
                    uint4 av[2 * PB];
                    if (MODE == 0) {
#pragma unroll
                        for (int j = 0; j < 2 * PB; ++j) av[j] = an[j];
                        const int nblk = G4 * q + PB * (pi + 1);  // first block of the next stage
#pragma unroll
                        for (int j = 0; j < 2 * PB; ++j)
                            an[j] = xrow && nblk < nb ? *reinterpret_cast<const uint4*>(xrow + nblk * 32 + 16 * j)
                                                      : make_uint4(0u, 0u, 0u, 0u);  // int8 zeros
                    }
                    if (s >= TS && !mbar_wait(&tile_free[s % TS], (s / TS - 1) & 1)) { ok = false; break; }
                    uint8_t* st = a_tile(s % TS, 0);
                    if (MODE == 0) {  // A: block b's 32 values -> chunks 0..3 of row `row`
#pragma unroll
                        for (int j = 0; j < 2 * PB; ++j)
                            int8x16_to_f16(av[j], st + (j >> 1) * (2 * TILE + 2 * STILE), row, 2 * (j & 1));
                    }
                    uint4 rv[2 * PB];
#pragma unroll
                    for (int j = 0; j < 2 * PB; ++j) {
                        int i, h;
                        chunk_of(pi, j, i, h);
                        rv[j] = *reinterpret_cast<const uint4*>(raw_half(rg, i, h));
                    }
#pragma unroll
                    for (int j = 0; j < 2 * PB; ++j) {
                        int i, h;
                        chunk_of(pi, j, i, h);
                        int8x16_to_f16(rv[j], st + (i % PB) * (2 * TILE + 2 * STILE) + TILE, row, 2 * h);
                    }
#pragma unroll
                    for (int b = 0; b < PB; ++b) {  // K element 0 of row `row` in both scale tiles
                        uint8_t* base = st + b * (2 * TILE + 2 * STILE) + 2 * TILE;
                        *reinterpret_cast<uint4*>(base + stile_row(row)) = make_uint4(xv[PB * pi + b], 0, 0, 0);
                        *reinterpret_cast<uint4*>(base + STILE + stile_row(row)) =
                            make_uint4(wv[PB * pi + b], 0, 0, 0);
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tile_full[s % TS]);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_free[slot]);
                w_cur = w_nxt;
                x_cur = x_nxt;
            }
        }
    } else if (warp == NEPI + NCONV) {
        // ---- MMA issuer: per block a fresh sumi accumulator (128 slots x 128 weight rows) and
        // the block's scale products (slot scale x row scale, one K = 16 MMA) next to it.
        // The whole warp walks the loop and waits; lane 0 issues the MMAs and their commits.
        const uint32_t id = idesc(TN);
        int s = 0, blk = 0;
        for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
            for (int p = 0; p < nb / PB; ++p, ++s) {
                const int ts = s % TS;
                if (!__all_sync(0xffffffffu, mbar_wait(&tile_full[ts], (s / TS) & 1))) { ok = false; break; }
                for (int b = 0; b < PB; ++b, ++blk) {
                    const int db = blk % DB;
                    if (blk >= DB && !__all_sync(0xffffffffu, mbar_wait(&d_free[db], (blk / DB - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (lane == 0) {
                        const uint8_t* at = a_tile(ts, b);
                        const uint32_t dcol = tmem + db * 2 * TN;
                        mma_f16(dcol, umma_desc(at, 0), umma_desc(at + TILE, 0), id, 0u);
                        mma_f16(dcol, umma_desc(at, 32), umma_desc(at + TILE, 32), id, 1u);
                        mma_f16(dcol + TN, umma_desc_plain(at + 2 * TILE), umma_desc_plain(at + 2 * TILE + STILE),
                                id, 0u);
                        mma_commit(&d_full[db]);
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (lane == 0) mma_commit(&tile_free[ts]);
                __syncwarp();
            }
        }
    } else {
        // ---- epilogue: slot 32 (w % 4) + lane; columns by w / 4 ----
        const int q4 = warp & 3, m = warp >> 2, srow = 32 * q4 + lane;
        const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
        const int c0 = MODE == 0 ? 32 * m : 64 * m, c1 = MODE == 0 ? 64 + 32 * m : 64 * m + 32;
        int blk = 0;
        for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
            const TileRef tr = tile_at(t);
            const bool live = 32 * q4 < tr.item.z;
            float acc[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) acc[j] = 0.0f;
            for (int kb = 0; kb < nb; ++kb, ++blk) {  // blocks in ascending order
                const int db = blk % DB;
                if (!mbar_wait(&d_full[db], (blk / DB) & 1)) { ok = false; break; }
                tc_fence_after();
                if (live) {
                    const uint32_t tb = tmem + lane_base + db * 2 * TN;
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq) {  // 16 columns at a time: sumi and scale product
                        const int cb = (qq < 2 ? c0 : c1) + 16 * (qq & 1);
                        uint32_t v[16], pr[16];
                        tmem_ld16_nw(tb + cb, v);
                        tmem_ld16_nw(tb + TN + cb, pr);
                        tmem_wait_ld();
                        float* ac = &acc[16 * qq];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const float x = __uint_as_float(v[e]), p = __uint_as_float(pr[e]);
                            if (FAST) ac[e] = __fmaf_rn(x, p, ac[e]);
                            else ac[e] = fadd(ac[e], fmul(x, p));
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&d_free[db]);
            }
            if (!ok || !live || srow >= tr.item.z) continue;
            const size_t slot = (size_t)tr.item.y + srow;
            if (MODE == 0) {
                // h rows f0 .. f0 + 31 of this slot: one Q8_0 block of the reference's h
                float h[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) h[j] = swiglu_ref(acc[j], acc[32 + j]);
                int8_t hq[32];
                const float sc = quant_block32(h, hq);
                const int f0 = tr.mt * 64 + 32 * m;
                uint4* dst = reinterpret_cast<uint4*>(a.h16 + slot * a.f + f0);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const __half2 p = __halves2half2(__int2half_rn(hq[8 * c + 2 * e]), __int2half_rn(hq[8 * c + 2 * e + 1]));
                        w[e] = *reinterpret_cast<const uint32_t*>(&p);
                    }
                    dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
                }
                a.hs[slot * (a.f / 32) + f0 / 32] = sc;
            } else {
                float4* dst = reinterpret_cast<float4*>(a.y + slot * a.d + tr.mt * TN + 64 * m);
#pragma unroll
                for (int j4 = 0; j4 < 16; ++j4)
                    dst[j4] = make_float4(acc[4 * j4], acc[4 * j4 + 1], acc[4 * j4 + 2], acc[4 * j4 + 3]);
            }
        }
    }
    if (!ok) atomicOr(err, PI_DEVERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(DB * 2 * TN) : "memory");
}

// Q8_0 weight rows for the TMA producer: gate/up [rows][d] bytes (box 64 B x 64 rows),
// lane-tiled down rows as {64 B, 8, cpq, rows/8} (box {16, 8, cpq, 16}).
bool q8_gateup_map(CUtensorMap* m, const PiMats& w) {
    const cuuint64_t dims[2] = {(cuuint64_t)w.cols, (cuuint64_t)(w.n * w.rows)};
    const cuuint64_t strides[1] = {(cuuint64_t)w.cols};
    const cuuint32_t box[2] = {64, 64};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}
bool q8_down_map(CUtensorMap* m, const PiMats& w) {
    const int64_t rows = w.n * w.rows, nch = w.cols / 16, cpq = nch / 4;
    const cuuint64_t dims[4] = {64, 8, (cuuint64_t)cpq, (cuuint64_t)(rows / 8)};
    const cuuint64_t strides[3] = {64, 512, (cuuint64_t)(8 * nch * 16)};
    const cuuint32_t box[4] = {16, 8, (cuuint32_t)cpq, 16};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, w.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}
// slot-major f16 activations [rows][cols]: 128 rows x 32 values per box, 64-byte swizzle
// (the K-major tile layout the MMA descriptors read)
bool act16_map(CUtensorMap* m, const __half* base, int64_t rows, int64_t cols) {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {32, 128};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}
}  // namespace

bool pi_prefill_q8_shape_ok(int64_t d, int64_t f) {
    // gate/up lane tiling needs d % 1024; down: 8 chunks per quarter row (f = 512) so that a
    // 4-block group is one 4-D box; 64-row gate/up and 128-row down tiles
    return d % 1024 == 0 && f == 512 && d % 128 == 0;
}

int pi_prefill_prepare_q8(pi_ctx* ctx, pi_moe_layer* L) {
    L->maps_ok = false;
    if (L->qtype != PI_QT_Q8_0 || !pi_prefill_q8_shape_ok(L->d, L->f)) return PI_OK;
    PiPrefillMaps& M = L->maps;
    bool ok = q8_gateup_map(&M.q[0][0], L->gate) && q8_gateup_map(&M.q[0][1], L->up) && q8_down_map(&M.q[0][2], L->down);
    if (ok && L->has_shared)
        ok = q8_gateup_map(&M.q[1][0], L->gate_sh) && q8_gateup_map(&M.q[1][1], L->up_sh) &&
             q8_down_map(&M.q[1][2], L->down_sh);
    if (!ok) return pi_set_error(ctx, PI_ERR_CUDA, "prefill Q8_0 GEMM: cuTensorMapEncodeTiled failed for the weights");
    L->maps_ok = true;
    return PI_OK;
}

int pi_prefill_experts_q8(pi_ctx* ctx, const pi_moe_layer* L, const ExpertArgs& a, int64_t max_items, int64_t T,
                          int64_t n_slots, int flags, cudaStream_t st) {
    if (L->qtype != PI_QT_Q8_0) return pi_set_error(ctx, PI_ERR_ARG, "prefill Q8_0 GEMM: Q8_0 weights only");
    if (!pi_prefill_q8_shape_ok(a.d, a.f) || (L->has_shared && L->f_sh != L->f))
        return pi_set_error(ctx, PI_ERR_ARG,
                            "prefill Q8_0 GEMM: n_embd must be a multiple of 1024 and the expert widths 512");
    if (!L->maps_ok) return pi_set_error(ctx, PI_ERR_CUDA, "prefill Q8_0 GEMM: weight tensor maps unavailable");
    if (!a.h16) return pi_set_error(ctx, PI_ERR_ARG, "prefill Q8_0 GEMM: slot buffers missing");
    (void)T;
    CUtensorMap mh;  // down reads h by TMA; gate/up gathers its slots' token rows in the converters
    if (!act16_map(&mh, a.h16, n_slots, a.f))
        return pi_set_error(ctx, PI_ERR_CUDA, "prefill Q8_0 GEMM: cuTensorMapEncodeTiled failed");
    const bool fast = (flags & PI_FWD_FAST_SUM) != 0;
    auto gu = fast ? k_moe_gemm_q8<0, true> : k_moe_gemm_q8<0, false>;
    auto dn = fast ? k_moe_gemm_q8<1, true> : k_moe_gemm_q8<1, false>;
    pi_smem_attr((const void*)gu, QSMEM);
    pi_smem_attr((const void*)dn, QSMEM);
    const int64_t sms = ctx->sm_count > 0 ? ctx->sm_count : 148;
    {
        PiProfScope ps(ctx, st, "k_gemm_q8_gateup");
        const unsigned g = (unsigned)std::min<int64_t>(max_items * (a.f / 64), sms);
        gu<<<g, QT, QSMEM, st>>>(a, L->maps, mh, nullptr, n_slots, ctx->dev_err);
    }
    {
        PiProfScope ps(ctx, st, "k_gemm_q8_down");
        const unsigned g = (unsigned)std::min<int64_t>(max_items * (a.d / TN), sms);
        dn<<<g, QT, QSMEM, st>>>(a, L->maps, mh, a.hs, n_slots, ctx->dev_err);
    }
    return pi_cuda_check(ctx, cudaGetLastError(), "prefill Q8_0 GEMM") ? PI_ERR_CUDA : PI_OK;
}
