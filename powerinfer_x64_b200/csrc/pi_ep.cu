// Expert-parallel data plane over NVLink peer memory (BASELINE config 5 at 2-8 GPUs).
//
// The reference has no multi-GPU path (it runs one process, model/mod.rs:1245-1571);
// this is the transport of the sharded layer. Every rank holds a block of device
// memory that its peers map through CUDA IPC; ranks write each other's blocks with
// plain stores over NVLink (no multicast, no collective library) and hand over with
// epoch flags:
//
//   push     each home token's Q8_0 row goes once to every rank that holds one of its
//            experts, with the local expert ids and gates of that rank
//            (one row per (token, destination rank));
//   experts  the destination runs its held experts over all received rows in one
//            grouped GEMM (and the shared expert over its own home tokens);
//   return   per received row the destination sums gate x expert output over the row's
//            experts (ascending) and writes that one partial row back to the home rank;
//   combine  the home rank adds the partial rows in ascending rank order (ranks hold
//            ascending expert ranges), then the gated shared expert, then x.
//
// Memory of rank R (parity p = epoch & 1, two epochs in flight):
//   rxq  [2][world][cap][d]    int8   rows rank src pushed to R
//   rxs  [2][world][cap][d/32] f32    their block scales
//   meta [2][world][cap][2k]   int32  local expert ids (-1 = none) then gate bits
//   rcnt [2][world]            int32  rows from each src
//   ret  [2][world][cap][d]    f32    partial rows rank dst returned for R's tokens
//   flag [4][world]            u64    recv (src pushed epoch e), ret (dst returned e),
//                                     ack_recv (dst read R's rows of e), ack_ret (home
//                                     read R's partials of e)
// A rank writes into a peer's parity-p region only after that peer acknowledged the
// epoch two before, so neither side ever waits on the other's later work. Every wait
// is bounded (about a second); a wait that gives up sets PI_DEVERR_TIMEOUT and returns.
#include "pi_common.cuh"
#include "pi_internal.h"

#include <cstring>

namespace {

enum { F_RECV = 0, F_RET = 1, F_ACK_RECV = 2, F_ACK_RET = 3 };
constexpr int EP_CHUNK = 256;  // tokens per position chunk (one per thread)

PI_DEV uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
PI_DEV void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Waits until flag[i] (this rank's memory) reaches `target` for every i < world
// (epochs only grow). Thread i watches rank i.
__global__ void k_ep_wait(const uint64_t* __restrict__ flags, int world, uint64_t target, uint32_t* __restrict__ err) {
    const int i = threadIdx.x;
    if (i >= world) return;
    const long long t0 = clock64();
    for (;;) {
        const uint64_t v = ld_acquire_sys(flags + i);
        if (v >= target) return;
        if (clock64() - t0 > (1ll << 31)) {
            atomicOr(err, PI_DEVERR_TIMEOUT);
            return;
        }
        __nanosleep(200);
    }
}

// Writes `value` into flag slot [which][me] of every peer (after this kernel's and the
// stream's earlier stores, made visible system-wide first).
__global__ void k_ep_signal(char* const* __restrict__ peers, size_t flag_off, int world, int me, int which,
                            uint64_t value, size_t rcnt_off, const int32_t* __restrict__ counts) {
    const int g = threadIdx.x;
    if (g >= world) return;
    char* pb = peers[g];
    if (counts) reinterpret_cast<int32_t*>(pb + rcnt_off)[me] = counts[g];
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint64_t*>(pb + flag_off) + (size_t)which * 64 + me, value);
}

// Per chunk of tokens: how many of them have an expert on each rank (cc[chunk][g]).
__global__ __launch_bounds__(EP_CHUNK) void k_ep_count(const int32_t* __restrict__ idx, int T, int k, int per_rank,
                                                       int world, int32_t* __restrict__ cc) {
    __shared__ int h[64];
    if (threadIdx.x < world) h[threadIdx.x] = 0;
    __syncthreads();
    const int t = blockIdx.x * EP_CHUNK + threadIdx.x;
    if (t < T) {
        uint64_t m = 0;
        for (int j = 0; j < k; ++j) m |= 1ull << (idx[(size_t)t * k + j] / per_rank);
        while (m) {
            const int g = __ffsll((long long)m) - 1;
            m &= m - 1;
            atomicAdd(&h[g], 1);
        }
    }
    __syncthreads();
    if (threadIdx.x < world) cc[(size_t)blockIdx.x * world + threadIdx.x] = h[threadIdx.x];
}

// Per rank an exclusive scan over chunks (cc becomes the chunk's first position) and
// the totals (rows this rank sends to each rank).
__global__ void k_ep_scan(int32_t* __restrict__ cc, int nchunk, int world, int32_t* __restrict__ total) {
    const int g = threadIdx.x;
    if (g >= world) return;
    int run = 0;
    for (int c = 0; c < nchunk; ++c) {
        const int v = cc[(size_t)c * world + g];
        cc[(size_t)c * world + g] = run;
        run += v;
    }
    total[g] = run;
}

// Position of each (token, rank) row in the rank's receive region, ascending tokens:
// dest_pos[t][g] = chunk start + the popcount of the chunk's earlier tokens bound for g
// (a bitmask per rank in shared memory); -1 where t has no expert on g.
__global__ __launch_bounds__(EP_CHUNK) void k_ep_pos(const int32_t* __restrict__ idx, int T, int k, int per_rank,
                                                     int world, const int32_t* __restrict__ cc,
                                                     int32_t* __restrict__ dest_pos) {
    __shared__ uint32_t mask[64 * (EP_CHUNK / 32)];
    for (int i = threadIdx.x; i < world * (EP_CHUNK / 32); i += EP_CHUNK) mask[i] = 0;
    __syncthreads();
    const int t = blockIdx.x * EP_CHUNK + threadIdx.x, w = threadIdx.x >> 5;
    const uint32_t bit = 1u << (threadIdx.x & 31);
    uint64_t m = 0;
    if (t < T)
        for (int j = 0; j < k; ++j) m |= 1ull << (idx[(size_t)t * k + j] / per_rank);
    for (uint64_t r = m; r;) {
        const int g = __ffsll((long long)r) - 1;
        r &= r - 1;
        atomicOr(&mask[g * (EP_CHUNK / 32) + w], bit);
    }
    __syncthreads();
    if (t >= T) return;
    for (int g = 0; g < world; ++g) {
        int pos = -1;
        if ((m >> g) & 1) {
            const uint32_t* mg = &mask[g * (EP_CHUNK / 32)];
            int r = __popc(mg[w] & (bit - 1));
            for (int x = 0; x < w; ++x) r += __popc(mg[x]);
            pos = cc[(size_t)blockIdx.x * world + g] + r;
        }
        dest_pos[(size_t)t * world + g] = pos;
    }
}

// One warp per (token, rank) row: the token's Q8_0 row, scales and the rank's expert
// ids / gates, stored straight into the rank's receive region.
__global__ __launch_bounds__(256) void k_ep_push(const int8_t* __restrict__ xq, const float* __restrict__ xs,
                                                 const int32_t* __restrict__ idx, const float* __restrict__ gates,
                                                 const int32_t* __restrict__ dest_pos, int T, int k, int per_rank,
                                                 int world, int me, int d, int64_t cap, int parity,
                                                 char* const* __restrict__ peers, size_t o_rxq, size_t o_rxs,
                                                 size_t o_meta) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= (int64_t)T * world) return;
    const int t = (int)(row / world), g = (int)(row % world);
    const int pos = dest_pos[row];
    if (pos < 0) return;
    char* pb = peers[g];
    const size_t r = ((size_t)parity * world + me) * cap + pos;
    const int4* src = reinterpret_cast<const int4*>(xq + (size_t)t * d);
    int4* dst = reinterpret_cast<int4*>(pb + o_rxq + r * d);
    for (int c = lane; c < d / 16; c += 32) dst[c] = src[c];
    const int4* ss = reinterpret_cast<const int4*>(xs + (size_t)t * (d / 32));
    int4* sd = reinterpret_cast<int4*>(pb + o_rxs + r * (d / 32) * 4);
    for (int c = lane; c < d / 128; c += 32) sd[c] = ss[c];
    if (lane < k) {
        int32_t* meta = reinterpret_cast<int32_t*>(pb + o_meta) + r * 2 * k;
        int32_t eid = -1;
        float gv = 0.0f;
        // this rank's experts among the token's (ascending), packed to the front
        int slot = 0;
        for (int j = 0; j < k; ++j) {
            const int e = idx[(size_t)t * k + j];
            if (e / per_rank == g) {
                if (slot == lane) {
                    eid = e - g * per_rank;
                    gv = gates[(size_t)t * k + j];
                }
                ++slot;
            }
        }
        meta[lane] = eid;
        meta[k + lane] = __float_as_int(gv);
    }
    __threadfence_system();
}

// Local expert ids of every received row ([world * cap][k]; rows past a source's
// count get -1, so the dispatch ignores them).
__global__ void k_ep_rows_idx(const int32_t* __restrict__ meta, const int32_t* __restrict__ rcnt, int world,
                              int64_t cap, int k, int32_t* __restrict__ eid) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)world * cap * k) return;
    const int64_t row = i / k;
    const int src = (int)(row / cap);
    const int64_t pos = row % cap;
    const int j = (int)(i % k);
    eid[i] = pos < rcnt[src] ? meta[row * 2 * k + j] : -1;
}

// Per received row: sum over its experts (ascending) of gate x expert output, from 0,
// written into the home rank's return region at the row's position.
__global__ __launch_bounds__(256) void k_ep_return(const float* __restrict__ y, const int32_t* __restrict__ slot_of,
                                                   const int32_t* __restrict__ meta, const int32_t* __restrict__ rcnt,
                                                   int world, int64_t cap, int k, int d, int me, int parity,
                                                   char* const* __restrict__ peers, size_t o_ret) {
    const int64_t row = blockIdx.x;
    const int src = (int)(row / cap);
    const int64_t pos = row % cap;
    if (pos >= rcnt[src]) return;
    const int32_t* mr = meta + row * 2 * k;
    float* dst = reinterpret_cast<float*>(peers[src] + o_ret) + (((size_t)parity * world + me) * cap + pos) * d;
    for (int c = 4 * threadIdx.x; c < d; c += 4 * blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < k; ++j) {
            if (mr[j] < 0) break;
            const float gv = __int_as_float(mr[k + j]);
            const float4 v = *reinterpret_cast<const float4*>(y + (size_t)slot_of[row * k + j] * d + c);
            acc.x = fadd(acc.x, fmul(gv, v.x));
            acc.y = fadd(acc.y, fmul(gv, v.y));
            acc.z = fadd(acc.z, fmul(gv, v.z));
            acc.w = fadd(acc.w, fmul(gv, v.w));
        }
        *reinterpret_cast<float4*>(dst + c) = acc;
    }
    __threadfence_system();
}

// out[t] = x[t] (residual) + ((partial of rank 0 + partial of rank 1 + ...) + s * y_sh[t]),
// partials in ascending rank order, which is ascending expert order.
__global__ __launch_bounds__(256) void k_ep_combine(const float* __restrict__ x, const float* __restrict__ ret,
                                                    const int32_t* __restrict__ dest_pos, const float* __restrict__ shscale,
                                                    const float* __restrict__ y, const int32_t* __restrict__ n_routed,
                                                    int has_shared, int T, int world, int64_t cap, int d, int parity,
                                                    int residual, float* __restrict__ out) {
    const int t = blockIdx.x;
    const int c = 4 * (blockIdx.y * blockDim.x + threadIdx.x);
    if (c >= d) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int g = 0; g < world; ++g) {
        const int pos = dest_pos[(size_t)t * world + g];
        if (pos < 0) continue;
        const float4 v = *reinterpret_cast<const float4*>(ret + (((size_t)parity * world + g) * cap + pos) * d + c);
        acc.x = fadd(acc.x, v.x);
        acc.y = fadd(acc.y, v.y);
        acc.z = fadd(acc.z, v.z);
        acc.w = fadd(acc.w, v.w);
    }
    if (has_shared) {
        const float s = shscale[t];
        const float4 v = *reinterpret_cast<const float4*>(y + ((size_t)*n_routed + t) * d + c);
        acc.x = fadd(acc.x, fmul(s, v.x));
        acc.y = fadd(acc.y, fmul(s, v.y));
        acc.z = fadd(acc.z, fmul(s, v.z));
        acc.w = fadd(acc.w, fmul(s, v.w));
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

size_t al(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace

struct pi_ep_comm {
    pi_ctx* ctx = nullptr;
    int rank = 0, world = 1, k = 0;
    int64_t cap = 0, d = 0;
    char* base = nullptr;
    size_t bytes = 0;
    size_t o_rxq = 0, o_rxs = 0, o_meta = 0, o_rcnt = 0, o_ret = 0, o_flag = 0;
    char* peer[PI_EP_MAX_WORLD] = {};
    bool mapped[PI_EP_MAX_WORLD] = {};
    char** peer_dev = nullptr;
    uint64_t epoch = 0;
    // rank-local scratch
    int32_t* dest_pos = nullptr;  // [cap][world]
    int32_t* cc = nullptr;        // [cap / EP_CHUNK + 1][world]
    int32_t* total = nullptr;     // [world]
    int32_t* eid = nullptr;       // [world * cap][k]
};

extern "C" int pi_ep_comm_create(pi_ctx* ctx, int32_t rank, int32_t world, int64_t max_tokens, int64_t n_embd,
                                 int32_t top_k, pi_ep_comm** out) {
    if (!ctx || !out) return PI_ERR_ARG;
    *out = nullptr;
    if (world < 1 || world > PI_EP_MAX_WORLD || rank < 0 || rank >= world || max_tokens < 1 || n_embd % 128 ||
        top_k < 1 || top_k > 32)
        return pi_set_error(ctx, PI_ERR_ARG, "ep comm: need 0 <= rank < world <= 64, n_embd % 128 == 0, k <= 32");
    cudaSetDevice(ctx->device);
    pi_ep_comm* c = new pi_ep_comm();
    c->ctx = ctx;
    c->rank = rank;
    c->world = world;
    c->k = top_k;
    c->cap = max_tokens;
    c->d = n_embd;
    const size_t W = world, cap = max_tokens, d = n_embd, k = top_k;
    size_t o = 0;
    c->o_rxq = o; o += al(2 * W * cap * d);
    c->o_rxs = o; o += al(2 * W * cap * (d / 32) * 4);
    c->o_meta = o; o += al(2 * W * cap * 2 * k * 4);
    c->o_rcnt = o; o += al(2 * W * 4);
    c->o_ret = o; o += al(2 * W * cap * d * 4);
    c->o_flag = o; o += al(4 * 64 * 8);
    c->bytes = o;
    int rc = PI_OK;
    if (pi_cuda_check(ctx, cudaMalloc(&c->base, c->bytes), "ep comm buffers")) rc = PI_ERR_OOM;
    if (!rc && pi_cuda_check(ctx, cudaMemset(c->base + c->o_flag, 0, 4 * 64 * 8), "ep flags")) rc = PI_ERR_CUDA;
    if (!rc && pi_cuda_check(ctx, cudaMemset(c->base + c->o_rcnt, 0, 2 * W * 4), "ep counts")) rc = PI_ERR_CUDA;
    const size_t nchunk = (cap + EP_CHUNK - 1) / EP_CHUNK + 1;
    if (!rc && pi_cuda_check(ctx, cudaMalloc(&c->dest_pos, cap * W * 4), "ep scratch")) rc = PI_ERR_OOM;
    if (!rc && pi_cuda_check(ctx, cudaMalloc(&c->cc, nchunk * W * 4), "ep scratch")) rc = PI_ERR_OOM;
    if (!rc && pi_cuda_check(ctx, cudaMalloc(&c->total, 64 * 4), "ep scratch")) rc = PI_ERR_OOM;
    if (!rc && pi_cuda_check(ctx, cudaMalloc(&c->eid, W * cap * k * 4), "ep scratch")) rc = PI_ERR_OOM;
    if (!rc && pi_cuda_check(ctx, cudaMalloc(&c->peer_dev, sizeof(char*) * PI_EP_MAX_WORLD), "ep peers")) rc = PI_ERR_OOM;
    if (rc) {
        pi_ep_comm_destroy(c);
        return rc;
    }
    c->peer[rank] = c->base;
    *out = c;
    return PI_OK;
}

extern "C" int pi_ep_comm_ipc_handle(pi_ep_comm* c, void* handle_out) {
    if (!c || !handle_out) return PI_ERR_ARG;
    cudaSetDevice(c->ctx->device);
    cudaIpcMemHandle_t h;
    if (pi_cuda_check(c->ctx, cudaIpcGetMemHandle(&h, c->base), "cudaIpcGetMemHandle")) return PI_ERR_CUDA;
    static_assert(sizeof(h) == PI_EP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof(h));
    return PI_OK;
}

extern "C" int pi_ep_comm_open(pi_ep_comm* c, const void* handles) {
    if (!c || !handles) return PI_ERR_ARG;
    cudaSetDevice(c->ctx->device);
    for (int g = 0; g < c->world; ++g) {
        if (g == c->rank || c->mapped[g]) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const char*>(handles) + (size_t)g * PI_EP_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        if (pi_cuda_check(c->ctx, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
            return PI_ERR_CUDA;
        c->peer[g] = static_cast<char*>(p);
        c->mapped[g] = true;
    }
    if (pi_cuda_check(c->ctx, cudaMemcpy(c->peer_dev, c->peer, sizeof(char*) * PI_EP_MAX_WORLD, cudaMemcpyHostToDevice),
                      "ep peers"))
        return PI_ERR_CUDA;
    return PI_OK;
}

extern "C" void pi_ep_comm_destroy(pi_ep_comm* c) {
    if (!c) return;
    if (c->ctx) cudaSetDevice(c->ctx->device);
    for (int g = 0; g < PI_EP_MAX_WORLD; ++g)
        if (c->mapped[g]) cudaIpcCloseMemHandle(c->peer[g]);
    cudaFree(c->base);
    cudaFree(c->dest_pos);
    cudaFree(c->cc);
    cudaFree(c->total);
    cudaFree(c->eid);
    cudaFree(c->peer_dev);
    delete c;
}

extern "C" int pi_ep_comm_debug_skip(pi_ep_comm* c, int32_t n) {
    if (!c || n < 0) return PI_ERR_ARG;
    c->epoch += (uint64_t)n;
    return PI_OK;
}

// One expert-parallel layer forward of this rank's T home tokens (see the top of the file).
extern "C" int pi_moe_ep_forward(pi_ctx* ctx, pi_moe_layer* L, pi_ep_comm* c, const float* x, int64_t T, float* out,
                                 int32_t flags, void* stream) {
    if (!ctx || !L || !c) return PI_ERR_ARG;
    if (T < 0 || T > c->cap || (T > 0 && (!x || !out)))
        return pi_set_error(ctx, PI_ERR_ARG, "ep forward: 0 <= T <= the comm's max_tokens, x and out required");
    if (L->qtype != PI_QT_Q8_0 || L->E % c->world || L->n_exp != L->E / c->world || L->k != c->k || L->d != c->d ||
        L->e_first != c->rank * L->n_exp)
        return pi_set_error(ctx, PI_ERR_ARG, "ep forward: the layer must hold this rank's E/world Q8_0 experts");
    if (((uintptr_t)x | (uintptr_t)out) & 15) return pi_set_error(ctx, PI_ERR_ARG, "ep forward: x, out 16-byte aligned");
    for (int g = 0; g < c->world; ++g)
        if (!c->peer[g]) return pi_set_error(ctx, PI_ERR_ARG, "ep forward: peers not opened (pi_ep_comm_open)");
    cudaStream_t st = (cudaStream_t)stream;
    const uint64_t e = ++c->epoch;
    const int p = (int)(e & 1), W = c->world, me = c->rank, k = c->k, d = (int)c->d, P = L->n_exp;
    const int64_t cap = c->cap;
    uint64_t* flags_local = reinterpret_cast<uint64_t*>(c->base + c->o_flag);

    // 1. routing of the home tokens (RMSNorm, router, top-k); Q8_0 rows kept
    const int64_t n_rows = W * cap;
    const size_t hb = al(pi_moe_ep_home_bytes(L, T, flags));
    char* scr;
    if (int rc = pi_scratch(ctx, st, hb + pi_moe_rows_multi_bytes(L, n_rows, k, T), &scr)) return rc;
    PiEpHome H;
    if (int rc = pi_moe_ep_home(ctx, L, x, T, flags, scr, &H, st)) return rc;
    const int nchunk = (int)((T + EP_CHUNK - 1) / EP_CHUNK);
    {
        PiProfScope ps(ctx, st, "k_ep_push");
        if (T > 0) {
            k_ep_count<<<(unsigned)nchunk, EP_CHUNK, 0, st>>>(H.idx, (int)T, k, P, W, c->cc);
            k_ep_scan<<<1, 64, 0, st>>>(c->cc, nchunk, W, c->total);
            k_ep_pos<<<(unsigned)nchunk, EP_CHUNK, 0, st>>>(H.idx, (int)T, k, P, W, c->cc, c->dest_pos);
        } else if (pi_cuda_check(ctx, cudaMemsetAsync(c->total, 0, 64 * 4, st), "ep totals")) {
            return PI_ERR_CUDA;
        }
        // the peers have read what this rank pushed two epochs ago
        if (e > 2) k_ep_wait<<<1, 64, 0, st>>>(flags_local + F_ACK_RECV * 64, W, e - 2, ctx->dev_err);
        if (T > 0) {
            const int64_t rows = T * W;
            k_ep_push<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(H.xq, H.xs, H.idx, H.gates, c->dest_pos, (int)T, k, P,
                                                                  W, me, d, cap, p, c->peer_dev, c->o_rxq, c->o_rxs,
                                                                  c->o_meta);
        }
        k_ep_signal<<<1, 64, 0, st>>>(c->peer_dev, c->o_flag, W, me, F_RECV, e, c->o_rcnt + (size_t)p * W * 4, c->total);
    }
    // 2. the rows every rank pushed here, through the held experts (+ the shared expert
    //    over the home tokens)
    {
        PiProfScope ps(ctx, st, "k_ep_wait");
        k_ep_wait<<<1, 64, 0, st>>>(flags_local + F_RECV * 64, W, e, ctx->dev_err);
    }
    const int32_t* rcnt = reinterpret_cast<const int32_t*>(c->base + c->o_rcnt) + (size_t)p * W;
    const int8_t* rxq = reinterpret_cast<const int8_t*>(c->base + c->o_rxq) + (size_t)p * W * cap * d;
    const float* rxs = reinterpret_cast<const float*>(c->base + c->o_rxs) + (size_t)p * W * cap * (d / 32);
    const int32_t* meta = reinterpret_cast<const int32_t*>(c->base + c->o_meta) + (size_t)p * W * cap * 2 * k;
    k_ep_rows_idx<<<(unsigned)((n_rows * k + 255) / 256), 256, 0, st>>>(meta, rcnt, W, cap, k, c->eid);
    PiRowsOut R;
    if (int rc = pi_moe_rows_multi_run(ctx, L, n_rows, k, rxq, rxs, c->eid, T, H.xq, H.xs, flags, scr + hb, &R, st))
        return rc;
    // 3. partial rows back to their home ranks (once the home ranks have combined the
    //    partials of two epochs ago)
    {
        PiProfScope ps(ctx, st, "k_ep_return");
        if (e > 2) k_ep_wait<<<1, 64, 0, st>>>(flags_local + F_ACK_RET * 64, W, e - 2, ctx->dev_err);
        k_ep_return<<<(unsigned)n_rows, 256, 0, st>>>(R.y, R.slot_of, meta, rcnt, W, cap, k, d, me, p, c->peer_dev,
                                                      c->o_ret);
        k_ep_signal<<<1, 64, 0, st>>>(c->peer_dev, c->o_flag, W, me, F_RET, e, 0, nullptr);
        k_ep_signal<<<1, 64, 0, st>>>(c->peer_dev, c->o_flag, W, me, F_ACK_RECV, e, 0, nullptr);
    }
    // 4. combine the returned partials of the home tokens
    {
        PiProfScope ps(ctx, st, "k_ep_combine");
        k_ep_wait<<<1, 64, 0, st>>>(flags_local + F_RET * 64, W, e, ctx->dev_err);
        if (T > 0)
            k_ep_combine<<<dim3((unsigned)T, (unsigned)((d + 1023) / 1024)), 256, 0, st>>>(
                x, reinterpret_cast<const float*>(c->base + c->o_ret), c->dest_pos, H.shscale, R.y, R.n_routed,
                L->has_shared ? 1 : 0, (int)T, W, cap, d, p, (flags & PI_FWD_RESIDUAL) ? 1 : 0, out);
        k_ep_signal<<<1, 64, 0, st>>>(c->peer_dev, c->o_flag, W, me, F_ACK_RET, e, 0, nullptr);
    }
    return pi_cuda_check(ctx, cudaGetLastError(), "ep forward") ? PI_ERR_CUDA : PI_OK;
}
