// Context, error handling, scratch arenas and the MoE-layer entry points.
#include "pi_common.cuh"
#include "pi_internal.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>

int pi_set_error(pi_ctx* ctx, int code, const std::string& msg) {
    if (ctx) {
        std::lock_guard<std::mutex> g(ctx->mu);
        ctx->last_error = msg;
    }
    return code;
}

int pi_cuda_check(pi_ctx* ctx, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return PI_OK;
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    return pi_set_error(ctx, e == cudaErrorMemoryAllocation ? PI_ERR_OOM : PI_ERR_CUDA, m);
}

// The dynamic shared-memory limit is an attribute of a kernel on one device, so
// it is raised once per (kernel, current device) and again whenever a launch
// needs more than was set; the record is shared by every thread of the process.
// The default limit covers static plus dynamic bytes up to 48 KB, so a request
// within 40 KB leaves any kernel here room for its static shared memory.
void pi_smem_attr(const void* fn, size_t bytes) {
    if (bytes <= 40 * 1024) return;
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    size_t& have = done[{fn, dev}];
    if (have >= bytes) return;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess) have = bytes;
    else cudaGetLastError();  // the launch that follows reports the failure
}

int pi_scratch(pi_ctx* ctx, cudaStream_t stream, size_t bytes, char** out) {
    std::lock_guard<std::mutex> g(ctx->mu);
    PiArena& a = ctx->arenas[stream];
    if (a.cap < bytes) {
        // A growing arena must not free memory that queued work on this
        // stream still reads: wait for the stream first.
        if (a.base) {
            cudaStreamSynchronize(stream);
            cudaFree(a.base);
            a.base = nullptr;
            a.cap = 0;
        }
        size_t cap = bytes + bytes / 4 + (1 << 20);
        if (cudaMalloc(&a.base, cap) != cudaSuccess) {
            cudaGetLastError();
            ctx->last_error = "scratch allocation of " + std::to_string(cap) + " bytes failed";
            return PI_ERR_OOM;
        }
        a.cap = cap;
    }
    *out = a.base;
    return PI_OK;
}

PiProfScope::PiProfScope(pi_ctx* c, cudaStream_t s, const char* nm) : ctx(c), st(s), name(nm) {
    if (!ctx->profiling) return;
    std::lock_guard<std::mutex> g(ctx->mu);
    for (auto& p : ctx->prof)
        if (p.name == nm) e = &p;
    if (!e) {
        ctx->prof.push_back(PiProfEntry{nm});
        e = &ctx->prof.back();
    }
    cudaEvent_t b, f;
    cudaEventCreate(&b);
    cudaEventCreate(&f);
    e->beg.push_back(b);
    e->end.push_back(f);
    cudaEventRecord(b, st);
}

PiProfScope::~PiProfScope() {
    if (e) cudaEventRecord(e->end.back(), st);
    // PI_DEBUG_SYNC=1: check and synchronise after every kernel of the layer
    // path and name the one that failed.
    static const bool debug_sync = [] {
        const char* v = std::getenv("PI_DEBUG_SYNC");
        return v && v[0] == '1';
    }();
    if (debug_sync) {
        cudaError_t err = cudaGetLastError();
        if (err == cudaSuccess) err = cudaStreamSynchronize(st);
        if (err != cudaSuccess) std::fprintf(stderr, "[pi debug] after %s: %s\n", name, cudaGetErrorString(err));
    }
}

extern "C" int pi_ctx_profile(pi_ctx* ctx, int enable) {
    if (!ctx) return PI_ERR_ARG;
    cudaDeviceSynchronize();
    std::lock_guard<std::mutex> g(ctx->mu);
    for (auto& p : ctx->prof) {
        for (auto ev : p.beg) cudaEventDestroy(ev);
        for (auto ev : p.end) cudaEventDestroy(ev);
    }
    ctx->prof.clear();
    ctx->profiling = enable != 0;
    return PI_OK;
}

extern "C" int pi_ctx_profile_read(pi_ctx* ctx, int max_entries, char* names, double* total_ms, int64_t* launches) {
    if (!ctx) return PI_ERR_ARG;
    cudaDeviceSynchronize();
    std::lock_guard<std::mutex> g(ctx->mu);
    int n = 0;
    for (auto& p : ctx->prof) {
        for (size_t i = 0; i < p.beg.size(); ++i) {
            float ms = 0;
            if (cudaEventElapsedTime(&ms, p.beg[i], p.end[i]) == cudaSuccess) p.total_ms += ms;
            cudaEventDestroy(p.beg[i]);
            cudaEventDestroy(p.end[i]);
        }
        p.launches += (long)p.beg.size();
        p.beg.clear();
        p.end.clear();
        if (n < max_entries) {
            std::strncpy(names + 32 * n, p.name.c_str(), 31);
            names[32 * n + 31] = 0;
            total_ms[n] = p.total_ms;
            launches[n] = p.launches;
        }
        ++n;
    }
    cudaGetLastError();
    return n;
}

extern "C" int pi_ctx_create(int device, pi_ctx** out) {
    if (!out) return PI_ERR_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return PI_ERR_CUDA;
    }
    if (cudaSetDevice(device) != cudaSuccess) return PI_ERR_CUDA;
    pi_ctx* c = new pi_ctx();
    c->device = device;
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
    if (cudaMalloc(&c->dev_err, sizeof(uint32_t)) != cudaSuccess || cudaMemset(c->dev_err, 0, 4) != cudaSuccess) {
        delete c;
        return PI_ERR_OOM;
    }
    *out = c;
    return PI_OK;
}

extern "C" void pi_ctx_destroy(pi_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    for (auto& kv : ctx->arenas)
        if (kv.second.base) cudaFree(kv.second.base);
    cudaFree(ctx->dev_err);
    delete ctx;
}

extern "C" const char* pi_last_error(const pi_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

extern "C" int pi_ctx_check(pi_ctx* ctx, void* stream) {
    if (!ctx) return PI_ERR_ARG;
    if (int rc = pi_cuda_check(ctx, cudaStreamSynchronize((cudaStream_t)stream), "stream sync")) return rc;
    uint32_t w = 0;
    if (int rc = pi_cuda_check(ctx, cudaMemcpy(&w, ctx->dev_err, 4, cudaMemcpyDeviceToHost), "read error word"))
        return rc;
    if (w) cudaMemset(ctx->dev_err, 0, 4);
    if (w & PI_DEVERR_INDEX) return pi_set_error(ctx, PI_ERR_INDEX, "index out of range");
    if (w & PI_DEVERR_TIMEOUT) return pi_set_error(ctx, PI_ERR_TIMEOUT, "device wait timed out");
    if (w) return pi_set_error(ctx, PI_ERR_ARG, "device-side shape error");
    return PI_OK;
}

extern "C" int pi_ctx_reserve(pi_ctx* ctx, void* stream, uint64_t bytes) {
    if (!ctx) return PI_ERR_ARG;
    char* p;
    return bytes ? pi_scratch(ctx, (cudaStream_t)stream, (size_t)bytes, &p) : PI_OK;
}

// --------------------------------------------------------------------------
// MoE layer
// --------------------------------------------------------------------------
extern "C" void pi_moe_layer_destroy(pi_moe_layer* L) {
    if (!L) return;
    for (void* p : L->allocs) cudaFree(p);
    delete L;
}

static int layer_create(pi_ctx* ctx, const pi_moe_layer_desc* D, int e_first, int n_exp, pi_moe_layer** out) {
    if (!ctx || !D || !out) return PI_ERR_ARG;
    *out = nullptr;
    if (e_first < 0 || n_exp < 1 || e_first + n_exp > D->n_expert)
        return pi_set_error(ctx, PI_ERR_ARG, "moe layer: held experts must lie in [0, n_expert)");
    if (D->qtype != PI_QT_Q8_0 && D->qtype != PI_QT_Q4_0)
        return pi_set_error(ctx, PI_ERR_ARG, "moe layer: expert weights must be Q8_0 or Q4_0");
    if (D->n_expert < 1 || D->n_expert > 512 || D->n_expert_used < 1 || D->n_expert_used > D->n_expert ||
        D->n_expert_used > 32)
        return pi_set_error(ctx, PI_ERR_ARG, "moe layer: need 1 <= k <= min(E, 32), E <= 512");
    if (!D->router || !D->gate_exps || !D->up_exps || !D->down_exps)
        return pi_set_error(ctx, PI_ERR_ARG, "moe layer: missing router or expert tensors");
    if (D->n_ff_exp != 128 && D->n_ff_exp != 256 && D->n_ff_exp != 512 && D->n_ff_exp != 1024)
        return pi_set_error(ctx, PI_ERR_ARG, "moe layer: expert width must be 128, 256, 512 or 1024");
    // the decode kernels are instantiated for these widths (Q8_0 gate/up by n_embd / 512,
    // Q4_0 by n_embd / 1024): any other n_embd would sum only part of each row
    if (D->qtype == PI_QT_Q8_0 ? (D->n_embd != 1024 && D->n_embd != 2048)
                               : (D->n_embd != 1024 && D->n_embd != 2048 && D->n_embd != 4096))
        return pi_set_error(ctx, PI_ERR_ARG,
                            D->qtype == PI_QT_Q8_0 ? "moe layer: Q8_0 n_embd must be 1024 or 2048"
                                                   : "moe layer: Q4_0 n_embd must be 1024, 2048 or 4096");
    const bool has_sh = D->gate_shexp && D->up_shexp && D->down_shexp;
    const int64_t f_sh = D->n_ff_shexp ? D->n_ff_shexp : D->n_ff_exp;
    if (has_sh && f_sh != D->n_ff_exp)
        return pi_set_error(ctx, PI_ERR_ARG, "moe layer: shared-expert width must equal the expert width");
    cudaSetDevice(ctx->device);
    pi_moe_layer* L = new pi_moe_layer();
    L->ctx = ctx;
    L->d = D->n_embd;
    L->f = D->n_ff_exp;
    L->f_sh = f_sh;
    L->E = D->n_expert;
    L->e_first = e_first;
    L->n_exp = n_exp;
    L->k = D->n_expert_used;
    L->qtype = D->qtype;
    L->has_shared = has_sh;
    L->has_shared_gate = has_sh && D->gate_inp_shexp;
    L->has_bias = D->router_bias != nullptr;
    const cudaMemcpyKind kind = D->src_on_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    const size_t rbytes = sizeof(float) * (size_t)(L->E + 1) * L->d;
    int rc = PI_OK;
    auto alloc = [&](void** p, size_t n) {
        if (rc) return;
        if (pi_cuda_check(ctx, cudaMalloc(p, n), "cudaMalloc")) rc = PI_ERR_OOM;
        else L->allocs.push_back(*p);
    };
    alloc((void**)&L->router, rbytes);
    if (!rc && pi_cuda_check(ctx, cudaMemset(L->router, 0, rbytes), "memset")) rc = PI_ERR_CUDA;
    if (!rc && pi_cuda_check(ctx, cudaMemcpy(L->router, D->router, sizeof(float) * L->E * L->d, kind), "router"))
        rc = PI_ERR_CUDA;
    if (!rc && L->has_shared_gate &&
        pi_cuda_check(ctx, cudaMemcpy(L->router + (size_t)L->E * L->d, D->gate_inp_shexp, sizeof(float) * L->d, kind),
                      "shared gate"))
        rc = PI_ERR_CUDA;
    if (L->has_bias) {
        alloc((void**)&L->bias, sizeof(float) * L->E);
        if (!rc && pi_cuda_check(ctx, cudaMemcpy(L->bias, D->router_bias, sizeof(float) * L->E, kind), "bias"))
            rc = PI_ERR_CUDA;
    }
    if (!rc) rc = pi_router_prepare(ctx, L);
    if (!rc) rc = pi_repack_mats(ctx, &L->gate, D->gate_exps, L->qtype, L->n_exp, L->f, L->d, D->src_on_host, &L->allocs);
    if (!rc) rc = pi_repack_mats(ctx, &L->up, D->up_exps, L->qtype, L->n_exp, L->f, L->d, D->src_on_host, &L->allocs);
    if (!rc) rc = pi_repack_mats(ctx, &L->down, D->down_exps, L->qtype, L->n_exp, L->d, L->f, D->src_on_host, &L->allocs);
    if (!rc) rc = pi_tile_down_mats(ctx, &L->down, &L->allocs);
    if (!rc && L->qtype == PI_QT_Q8_0) rc = pi_tile_gateup_mats(ctx, &L->gate, &L->allocs);
    if (!rc && L->qtype == PI_QT_Q8_0) rc = pi_tile_gateup_mats(ctx, &L->up, &L->allocs);
    if (has_sh) {
        if (!rc) rc = pi_repack_mats(ctx, &L->gate_sh, D->gate_shexp, L->qtype, 1, f_sh, L->d, D->src_on_host, &L->allocs);
        if (!rc) rc = pi_repack_mats(ctx, &L->up_sh, D->up_shexp, L->qtype, 1, f_sh, L->d, D->src_on_host, &L->allocs);
        if (!rc) rc = pi_repack_mats(ctx, &L->down_sh, D->down_shexp, L->qtype, 1, L->d, f_sh, D->src_on_host, &L->allocs);
        if (!rc) rc = pi_tile_down_mats(ctx, &L->down_sh, &L->allocs);
        if (!rc && L->qtype == PI_QT_Q8_0) rc = pi_tile_gateup_mats(ctx, &L->gate_sh, &L->allocs);
        if (!rc && L->qtype == PI_QT_Q8_0) rc = pi_tile_gateup_mats(ctx, &L->up_sh, &L->allocs);
    }
    if (!rc) rc = L->qtype == PI_QT_Q8_0 ? pi_prefill_prepare_q8(ctx, L) : pi_prefill_prepare(ctx, L);
    if (rc) {
        pi_moe_layer_destroy(L);
        return rc;
    }
    *out = L;
    return PI_OK;
}

extern "C" int pi_moe_layer_create(pi_ctx* ctx, const pi_moe_layer_desc* D, pi_moe_layer** out) {
    return layer_create(ctx, D, 0, D ? D->n_expert : 0, out);
}

extern "C" int pi_moe_layer_create_ep(pi_ctx* ctx, const pi_moe_layer_desc* D, int32_t first_expert, int32_t n_local,
                                      pi_moe_layer** out) {
    if (D && D->qtype != PI_QT_Q8_0 && ctx)
        return pi_set_error(ctx, PI_ERR_ARG, "expert-parallel layer: Q8_0 experts only");
    return layer_create(ctx, D, first_expert, n_local, out);
}

static int moe_common(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, float* out, int flags,
                      int32_t* idx, float* gates, int32_t* counts, int32_t* offsets, int32_t* perm, void* stream) {
    if (!ctx || !L) return PI_ERR_ARG;
    if (T < 0 || (T > 0 && !x)) return pi_set_error(ctx, PI_ERR_ARG, "moe: bad token batch");
    if (T == 0) return PI_OK;
    if (T > (1 << 20)) return pi_set_error(ctx, PI_ERR_ARG, "moe: T too large");
    if (((uintptr_t)x | (uintptr_t)out) & 15)  // the kernels read and write token rows with 16-byte accesses
        return pi_set_error(ctx, PI_ERR_ARG, "moe: x and out must be 16-byte aligned");
    if (out && L->n_exp != L->E)
        return pi_set_error(ctx, PI_ERR_ARG, "moe forward: the layer holds a subset of the experts (use the pi_moe_ep_* calls)");
    cudaStream_t st = (cudaStream_t)stream;
    char* scr;
    if (int rc = pi_scratch(ctx, st, pi_moe_scratch_bytes(L, T, flags), &scr)) return rc;
    return pi_moe_run(ctx, L, x, T, out, flags, idx, gates, counts, offsets, perm, scr, st);
}

extern "C" int pi_moe_ep_route(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, int32_t flags, int32_t world,
                               int32_t* idx, float* gates, float* shscale, int8_t* xq, float* xs, int32_t* send_counts,
                               int8_t* send_xq, float* send_xs, int32_t* send_eid, int32_t* slot_row, void* stream) {
    if (!ctx || !L) return PI_ERR_ARG;
    if (T < 0 || (T > 0 && !x) || world < 1 || world > 64 || L->E % world || L->n_exp != L->E / world ||
        L->qtype != PI_QT_Q8_0)
        return pi_set_error(ctx, PI_ERR_ARG, "ep route: Q8_0 layer holding E/world experts, 1 <= world <= 64");
    if (T > (1 << 20)) return pi_set_error(ctx, PI_ERR_ARG, "ep route: T too large");
    cudaStream_t st = (cudaStream_t)stream;
    if (T == 0) {
        return pi_cuda_check(ctx, cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * world, st), "ep counts")
                   ? PI_ERR_CUDA
                   : PI_OK;
    }
    const int f = (flags & (PI_FWD_RMSNORM | PI_FWD_RESIDUAL)) | PI_FWD_FORCE_GEMV | PI_FWD_KEEP_Q8;
    char* scr;
    // + the send-order token list and the per-chunk counts
    const size_t n = (size_t)T * L->k, nchunk = (n + 1023) / 1024;
    if (int rc = pi_scratch(ctx, st, pi_moe_scratch_bytes(L, T, f) + 512 + sizeof(int32_t) * (n + 64 + nchunk * world), &scr))
        return rc;
    return pi_moe_ep_route_run(ctx, L, x, T, f, world, idx, gates, shscale, xq, xs, send_counts, send_xq, send_xs,
                               send_eid, slot_row, scr, st);
}

extern "C" int pi_moe_experts_q8(pi_ctx* ctx, pi_moe_layer* L, int64_t n_rows, const int8_t* xq, const float* xs,
                                 const int32_t* eid, float* y, void* stream) {
    if (!ctx || !L) return PI_ERR_ARG;
    if (n_rows < 0 || n_rows > (1 << 24) || L->qtype != PI_QT_Q8_0 || (!eid && !L->has_shared))
        return pi_set_error(ctx, PI_ERR_ARG, "experts: Q8_0 layer; eid = NULL needs a shared expert");
    if (n_rows == 0) return PI_OK;
    cudaStream_t st = (cudaStream_t)stream;
    char* scr;
    if (int rc = pi_scratch(ctx, st, pi_moe_rows_scratch_bytes(L, n_rows), &scr)) return rc;
    return pi_moe_rows_run(ctx, L, n_rows, xq, xs, eid, y, scr, st);
}

extern "C" int pi_moe_ep_combine(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, int32_t flags,
                                 const float* gates, const float* shscale, const int32_t* slot_row, const float* y_back,
                                 const float* y_shared, float* out, void* stream) {
    if (!ctx || !L) return PI_ERR_ARG;
    if (T < 0) return pi_set_error(ctx, PI_ERR_ARG, "ep combine: bad token batch");
    if (T == 0) return PI_OK;
    if (((uintptr_t)x | (uintptr_t)out | (uintptr_t)y_back | (uintptr_t)y_shared) & 15)
        return pi_set_error(ctx, PI_ERR_ARG, "ep combine: x, out and the expert rows must be 16-byte aligned");
    return pi_moe_ep_combine_run(ctx, L, x, T, flags, gates, shscale, slot_row, y_back, y_shared, out,
                                 (cudaStream_t)stream);
}

extern "C" int pi_moe_route(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, int32_t* idx, float* gates,
                            int32_t* counts, int32_t* offsets, int32_t* perm, void* stream) {
    return moe_common(ctx, L, x, T, nullptr, 0, idx, gates, counts, offsets, perm, stream);
}

extern "C" int pi_moe_forward(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, float* out, int32_t flags,
                              void* stream) {
    if (!out && T > 0) return pi_set_error(ctx, PI_ERR_ARG, "moe: null output");
    return moe_common(ctx, L, x, T, out, flags, nullptr, nullptr, nullptr, nullptr, nullptr, stream);
}

extern "C" int pi_moe_forward_routed(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, float* out,
                                     int32_t flags, int32_t* idx, float* gates, int32_t* counts, int32_t* offsets,
                                     int32_t* perm, void* stream) {
    if (!out && T > 0) return pi_set_error(ctx, PI_ERR_ARG, "moe: null output");
    return moe_common(ctx, L, x, T, out, flags, idx, gates, counts, offsets, perm, stream);
}
