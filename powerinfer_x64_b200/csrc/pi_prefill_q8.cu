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
// fresh accumulator; a stage carries PB = 2 blocks (one handshake for both) into
// the two column halves of one of DB TMEM buffers; epilogue warps apply each
// block's scales and add it to f32 registers in block order, so each output is
// the reference's own sequence of roundings. The gate/up kernel stacks 64 gate
// rows over the same 64 up rows in one 128-row tile, applies the reference's
// SwiGLU and quantises h to Q8_0 per 32 rows (a warp's 32 lanes), exactly as
// the reference's ffn_swiglu_q does before its down matvec (quant/mod.rs:1184-1249);
// the down kernel writes y.
//
// Data movement (TMA, no multicast) runs in groups of 4 blocks (128 K bytes):
// weight rows of both lane-tiled layouts as 2-D / 4-D boxes, the gate/up
// token rows by tile::gather4 from the token-major Q8_0 activations, the down
// kernel's slot-major h rows as one box.
//
// Warp roles (QT = 832 threads, one CTA per SM):
//   0-15  epilogue: warp w owns TMEM lanes 32 (w % 4) .. +31 (weight rows) and
//         slot columns 32 (w / 4) .. +31;
//   16-23 converters: thread c < 128 converts weight row c, c >= 128 slot row
//         c - 128, of each block from the raw group into an f16 tile row
//         (64-byte swizzled K-major) and publishes the row's block scale;
//   24    MMA issuer;  25 TMA producer.
// Every mbarrier wait is bounded and reports PI_DEVERR_TIMEOUT.
#include "pi_tc.cuh"
// pi_tc.cuh (pi_common.cuh) comes first: it names the quant types that pi_moe.h defines as macros
#include "pi_internal.h"

namespace {
using namespace pitc;

constexpr int QN = PI_GEMM_NT_Q8;  // slots per item (max MMA N)
constexpr int NEPI = 16, NCONV = 8;
constexpr int QT = (NEPI + NCONV + 2) * 32;
constexpr int G4 = 4;              // blocks per raw group
constexpr int RG = 2;              // raw groups in flight
constexpr int PB = 2;              // blocks per stage (one handshake)
constexpr int TS = 4;              // f16 tile stages of PB blocks
constexpr int DB = 2;              // TMEM buffers of PB x QN columns
constexpr int SB = 4;              // block-scale buffers (stages)
constexpr int TILE = 128 * 64;     // 128 rows x 32 f16
constexpr int STAGE = PB * 2 * TILE;  // {W tile, X tile} per block
constexpr int RAWW = 128 * G4 * 32;  // weight rows of a group (16 KB)
constexpr int RAWG = 2 * RAWW;       // + activation rows
static_assert(G4 == 2 * PB, "a raw group fills two stages");
constexpr size_t QSMEM = (size_t)RG * RAWG + (size_t)TS * STAGE + 1024;

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

// MODE 0: gate/up (+ SwiGLU, Q8_0 h); MODE 1: down (y).
template <int MODE>
__global__ __launch_bounds__(QT, 1) void k_moe_gemm_q8(ExpertArgs a, const __grid_constant__ PiPrefillMaps wm,
                                                       const __grid_constant__ CUtensorMap mx, uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* tiles = sm;              // TS stages of PB x {W tile, X tile}
    uint8_t* raws = sm + TS * STAGE;  // RG groups of {W rows, X rows}
    __shared__ __align__(8) uint64_t tile_full[TS], tile_free[TS], d_full[DB], d_free[DB], scl_full[SB], scl_free[SB];
    __shared__ __align__(8) uint64_t raw_full[RG], raw_free[RG];
    __shared__ __align__(16) float s_dw[SB][PB][128];
    __shared__ __align__(16) float s_dx[SB][PB][QN];
    __shared__ uint32_t s_tmem;
    __shared__ int s_row[QN];  // gate/up: token of each slot column; down: slot
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int it = blockIdx.y;
    if (it >= *a.n_items) return;
    const int4 item = a.items[it];
    const bool sh = item.x == a.E;
    const int K = MODE == 0 ? a.d : a.f;
    const int nb = K / 32, ng = nb / G4, np = nb / PB;
    const int nn = (item.z + 15) & ~15;

    if (tid == 0) {
        for (int i = 0; i < TS; ++i) {
            mbar_init(&tile_full[i], NCONV);
            mbar_init(&tile_free[i], 1);
        }
        for (int i = 0; i < DB; ++i) {
            mbar_init(&d_full[i], 1);
            mbar_init(&d_free[i], NEPI);
        }
        for (int i = 0; i < SB; ++i) {
            mbar_init(&scl_full[i], NCONV);
            mbar_init(&scl_free[i], NEPI);
        }
        for (int i = 0; i < RG; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_free[i], NCONV);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int r = tid; r < QN; r += QT) {
        const int sl = item.y + (r < item.z ? r : 0);
        s_row[r] = MODE == 1 ? sl : (sl < a.n_routed ? a.perm[sl] : sl - a.n_routed);
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(DB * PB * QN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ok = true;
    const int mrow = sh ? 0 : item.x * (MODE == 0 ? a.f : a.d);  // expert's first row in its family

    if (warp == NEPI + NCONV + 1) {
        // ---- TMA producer: group q -> raw slot q % RG once the converters released q - RG ----
        for (int q = 0; q < ng; ++q) {
            const int slot = q % RG, use = q / RG;
            int w_ok = 1;
            if (lane == 0) {
                if (use > 0 && !mbar_wait(&raw_free[slot], (use - 1) & 1)) w_ok = 0;
                else mbar_expect_tx(&raw_full[slot], RAWG);
            }
            if (!__shfl_sync(0xffffffffu, w_ok, 0)) { ok = false; break; }
            uint8_t* rw = raws + slot * RAWG;
            uint8_t* rx = rw + RAWW;
            if (MODE == 0) {
                if (lane == 0) {
                    // lane-tiled gate/up rows: half h of block B at ((B/32)*64 + h*32 + B%32) * 16 bytes,
                    // so the first halves of blocks 4q..4q+3 are 64 contiguous bytes, the second ones +512
                    const int b0 = G4 * q, x0 = ((b0 >> 5) * 64 + (b0 & 31)) * 16;
                    const int r0 = mrow + blockIdx.x * 64;
                    const CUtensorMap* mg = sh ? &wm.q[1][0] : &wm.q[0][0];
                    const CUtensorMap* mu = sh ? &wm.q[1][1] : &wm.q[0][1];
                    tma_load_2d(rw, mg, x0, r0, &raw_full[slot]);
                    tma_load_2d(rw + 64 * 64, mg, x0 + 512, r0, &raw_full[slot]);
                    tma_load_2d(rw + 2 * 64 * 64, mu, x0, r0, &raw_full[slot]);
                    tma_load_2d(rw + 3 * 64 * 64, mu, x0 + 512, r0, &raw_full[slot]);
                }
                __syncwarp();
                const int* tk = &s_row[4 * lane];  // 32 lanes x 4 rows = the 128 slot rows
                tma_gather4(rx + lane * 4 * 128, &mx, q * 128, tk[0], tk[1], tk[2], tk[3], &raw_full[slot]);
            } else if (lane == 0) {
                // lane-tiled down rows: chunk j of row r at ((r/8)*8*nch + (j%cpq)*32 + (r%8)*4 + j/cpq) * 16,
                // blocks 4q..4q+3 = chunks 8q..8q+7 = all j%cpq with j/cpq = q (cpq = 8)
                const CUtensorMap* md = sh ? &wm.q[1][2] : &wm.q[0][2];
                tma_load_4d(rw, md, q * 16, 0, 0, (mrow + blockIdx.x * 128) >> 3, &raw_full[slot]);
                tma_load_2d(rx, &mx, q * 128, item.y, &raw_full[slot]);
            }
        }
    } else if (warp >= NEPI && warp < NEPI + NCONV) {
        // ---- converters: thread c < 128 converts weight row c, c >= 128 slot row c - 128 ----
        const int c = tid - NEPI * 32, row = c & 127;
        const bool isx = c >= 128;
        // this row's block scales, 4 per group, loaded one group ahead
        const void* scp;
        if (!isx) {
            const __half* wd;
            int wr;
            if (MODE == 0) {
                const bool up = row >= 64;
                wd = up ? (sh ? a.usd : a.ud) : (sh ? a.gsd : a.gd);
                wr = mrow + blockIdx.x * 64 + (row & 63);
            } else {
                wd = sh ? a.dsd : a.dd;
                wr = mrow + blockIdx.x * 128 + row;
            }
            scp = wd + (size_t)wr * nb;
        } else {
            scp = (MODE == 0 ? a.xs + (size_t)s_row[row] * nb : a.hs + (size_t)s_row[row] * nb);
        }
        auto load_sc = [&](int q, float (&v)[G4]) {
            if (isx) {
                const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(scp) + G4 * q);
                v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
            } else {
                const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(scp) + G4 * q);
                const __half2 h0 = *reinterpret_cast<const __half2*>(&h.x), h1 = *reinterpret_cast<const __half2*>(&h.y);
                v[0] = __low2float(h0); v[1] = __high2float(h0); v[2] = __low2float(h1); v[3] = __high2float(h1);
            }
        };
        // raw position of this row's 32 bytes of block i (two 16-byte halves)
        auto raw_half = [&](const uint8_t* rg, int i, int h) -> const uint8_t* {
            if (isx) return rg + RAWW + row * 128 + 32 * i + 16 * h;
            if (MODE == 0) return rg + (row >> 6) * 2 * 64 * 64 + h * 64 * 64 + (row & 63) * 64 + 16 * i;
            return rg + (row >> 3) * 1024 + (2 * i + h) * 128 + (row & 7) * 16;  // [r/8][chunk][r%8][16 B]
        };
        // Chunk j (0..7) of this row's group -> (block i, half h). The order is rotated per row
        // so that the 32 lanes of a load touch distinct shared-memory banks: activation rows
        // are 128 bytes apart (chunk 2i + h), gate/up weight rows 64 bytes apart (chunk i of
        // half h), down weight rows already interleave 8 rows per 128 bytes.
        auto chunk_of = [&](int j, int& i, int& h) {
            if (isx) {
                const int k = (j + row) & 7;
                i = k >> 1;
                h = k & 1;
            } else if (MODE == 0) {
                i = (j + (row >> 1)) & 3;
                h = j >> 2;
            } else {
                i = j >> 1;
                h = j & 1;
            }
        };
        float sc_cur[G4], sc_nxt[G4];
        load_sc(0, sc_cur);
        for (int q = 0; q < ng && ok; ++q) {
            const int slot = q % RG;
            if (q + 1 < ng) load_sc(q + 1, sc_nxt);
            if (!mbar_wait(&raw_full[slot], (q / RG) & 1)) { ok = false; break; }
#pragma unroll
            for (int pi = 0; pi < G4 / PB; ++pi) {  // the group's stages: tiles and scale buffers free
                const int g = (G4 / PB) * q + pi;
                if (g >= TS && !mbar_wait(&tile_free[g % TS], (g / TS - 1) & 1)) ok = false;
                if (g >= SB && !mbar_wait(&scl_free[g % SB], (g / SB - 1) & 1)) ok = false;
            }
            if (!ok) break;
            const uint8_t* rg = raws + slot * RAWG;
#pragma unroll
            for (int j = 0; j < 2 * G4; ++j) {
                int i, h;
                chunk_of(j, i, h);
                const int g = (G4 / PB) * q + i / PB;
                int8x16_to_f16(*reinterpret_cast<const uint4*>(raw_half(rg, i, h)),
                               tiles + (g % TS) * STAGE + (i % PB) * 2 * TILE + (isx ? TILE : 0), row, 2 * h);
            }
#pragma unroll
            for (int i = 0; i < G4; ++i) {
                const int sb = ((G4 / PB) * q + i / PB) % SB;
                (isx ? s_dx[sb][i % PB] : s_dw[sb][i % PB])[row] = sc_cur[i];
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
#pragma unroll
                for (int pi = 0; pi < G4 / PB; ++pi) {
                    const int g = (G4 / PB) * q + pi;
                    mbar_arrive(&tile_full[g % TS]);
                    mbar_arrive(&scl_full[g % SB]);
                }
                mbar_arrive(&raw_free[slot]);
            }
#pragma unroll
            for (int i = 0; i < G4; ++i) sc_cur[i] = sc_nxt[i];
        }
    } else if (warp == NEPI + NCONV) {
        // ---- MMA issuer ----
        if (lane == 0) {
            const uint32_t id = idesc(nn);
            for (int g = 0; g < np; ++g) {
                const int ts = g % TS, db = g % DB;
                if (!mbar_wait(&tile_full[ts], (g / TS) & 1) ||
                    (g >= DB && !mbar_wait(&d_free[db], (g / DB - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int b = 0; b < PB; ++b) {  // block b -> a fresh accumulator in column half b
                    const uint8_t* wt = tiles + ts * STAGE + b * 2 * TILE;
                    const uint32_t dcol = tmem + (db * PB + b) * QN;
                    mma_f16(dcol, umma_desc(wt, 0), umma_desc(wt + TILE, 0), id, 0u);
                    mma_f16(dcol, umma_desc(wt, 32), umma_desc(wt + TILE, 32), id, 1u);
                }
                mma_commit(&tile_free[ts]);
                mma_commit(&d_full[db]);
            }
        }
    } else {
        // ---- epilogue: rows 32 (w % 4) + lane, slot columns 32 (w / 4) .. +31 ----
        const int q4 = warp & 3, cg = warp >> 2, rl = 32 * q4 + lane;
        const bool live = 32 * cg < item.z;
        const uint32_t lane_base = (uint32_t)(32 * q4) << 16;
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
        for (int g = 0; g < np; ++g) {
            const int db = g % DB, sb = g % SB;
            if (!mbar_wait(&d_full[db], (g / DB) & 1) || !mbar_wait(&scl_full[sb], (g / SB) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (live) {
#pragma unroll
                for (int b = 0; b < PB; ++b) {  // the stage's blocks in ascending order
                    const float dw = s_dw[sb][b][rl];
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        float v[16];
                        tmem_ld16(tmem + lane_base + (db * PB + b) * QN + 32 * cg + 16 * hh, v);
#pragma unroll
                        for (int j4 = 0; j4 < 4; ++j4) {
                            const float4 dx = *reinterpret_cast<const float4*>(&s_dx[sb][b][32 * cg + 16 * hh + 4 * j4]);
                            float* ac = &acc[16 * hh + 4 * j4];
                            ac[0] = fadd(ac[0], fmul(v[4 * j4], fmul(dw, dx.x)));
                            ac[1] = fadd(ac[1], fmul(v[4 * j4 + 1], fmul(dw, dx.y)));
                            ac[2] = fadd(ac[2], fmul(v[4 * j4 + 2], fmul(dw, dx.z)));
                            ac[3] = fadd(ac[3], fmul(v[4 * j4 + 3], fmul(dw, dx.w)));
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&d_free[db]);
                mbar_arrive(&scl_free[sb]);
            }
        }
        if (MODE == 0) {
            // up rows (quarters 2, 3) hand their sums to the gate rows through shared memory
            float* s_up = reinterpret_cast<float*>(raws);  // the raw ring is idle now
            asm volatile("bar.sync 1, %0;" ::"n"(NEPI * 32) : "memory");
            if (q4 >= 2 && live) {
#pragma unroll
                for (int j = 0; j < 32; ++j) s_up[(32 * (q4 - 2) + lane) * (QN + 1) + 32 * cg + j] = acc[j];
            }
            asm volatile("bar.sync 1, %0;" ::"n"(NEPI * 32) : "memory");
            if (q4 < 2 && live) {
                const int f0 = blockIdx.x * 64 + 32 * q4;  // first h row of this warp = one Q8_0 block
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(DB * PB * QN) : "memory");
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
// int8 activations [rows][cols]: gate/up gathers 128-byte rows (box one row high),
// down loads 128 slot rows x 128 bytes
bool q8_act_map(CUtensorMap* m, const int8_t* base, int64_t rows, int64_t cols, int box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols};
    const cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
    return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
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
                          int64_t n_slots, cudaStream_t st) {
    if (L->qtype != PI_QT_Q8_0) return pi_set_error(ctx, PI_ERR_ARG, "prefill Q8_0 GEMM: Q8_0 weights only");
    if (!pi_prefill_q8_shape_ok(a.d, a.f) || (L->has_shared && L->f_sh != L->f))
        return pi_set_error(ctx, PI_ERR_ARG,
                            "prefill Q8_0 GEMM: n_embd must be a multiple of 1024 and the expert widths 512");
    if (!L->maps_ok) return pi_set_error(ctx, PI_ERR_CUDA, "prefill Q8_0 GEMM: weight tensor maps unavailable");
    static_assert((size_t)RG * RAWG >= (size_t)64 * (QN + 1) * 4, "the up-row exchange fits in the raw ring");
    CUtensorMap mxg, mhq;
    if (!q8_act_map(&mxg, a.xq, T, a.d, 1) || !q8_act_map(&mhq, a.hq, n_slots, a.f, 128))
        return pi_set_error(ctx, PI_ERR_CUDA, "prefill Q8_0 GEMM: cuTensorMapEncodeTiled failed");
    pi_smem_attr((const void*)k_moe_gemm_q8<0>, QSMEM);
    pi_smem_attr((const void*)k_moe_gemm_q8<1>, QSMEM);
    {
        PiProfScope ps(ctx, st, "k_gemm_q8_gateup");
        k_moe_gemm_q8<0><<<dim3((unsigned)(a.f / 64), (unsigned)max_items), QT, QSMEM, st>>>(a, L->maps, mxg,
                                                                                           ctx->dev_err);
    }
    {
        PiProfScope ps(ctx, st, "k_gemm_q8_down");
        k_moe_gemm_q8<1><<<dim3((unsigned)(a.d / 128), (unsigned)max_items), QT, QSMEM, st>>>(a, L->maps, mhq,
                                                                                            ctx->dev_err);
    }
    return pi_cuda_check(ctx, cudaGetLastError(), "prefill Q8_0 GEMM") ? PI_ERR_CUDA : PI_OK;
}
