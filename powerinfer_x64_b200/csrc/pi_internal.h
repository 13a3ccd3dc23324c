// Internal (non-ABI) declarations shared by the library's translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <deque>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/pi_moe.h"

// One quantised matrix family stored structure-of-arrays in HBM:
//   Q8_0: q = int8  [n][rows][cols]        d = f16 [n][rows][cols/32]
//   Q4_0: q = uint8 [n][rows][cols/2]      d = f16 [n][rows][cols/32]
//         (the 16 nibble bytes of each GGUF block kept in their original
//          order: byte i low nibble = element 2i, high nibble = 2i+1)
//   F32 : q = float [n][rows][cols]        d = null
// Rows are 16-byte aligned whenever cols % 32 == 0 (Q8_0) or % 64 == 0 (Q4_0),
// which the layer constructor requires, so kernels use 16-byte vector loads.
struct PiMats {
    int qtype = PI_QT_F32;
    int64_t n = 0, rows = 0, cols = 0;
    void* q = nullptr;
    __half* d = nullptr;
    int64_t q_row_bytes() const {
        return qtype == PI_QT_Q8_0 ? cols : (qtype == PI_QT_Q4_0 ? cols / 2 : cols * 4);
    }
    int64_t q_mat_bytes() const { return q_row_bytes() * rows; }
    int64_t d_mat_elems() const { return rows * (cols / 32); }
};

// TMA descriptors of a Q4_0 layer's weights for the prefill GEMM:
// [routed / shared][gate, up, down] raw nibbles and f16 scales.
struct __align__(64) PiPrefillMaps {
    CUtensorMap q[2][3];
    CUtensorMap d[2][3];
};

struct pi_moe_layer {
    pi_ctx* ctx = nullptr;
    int64_t d = 0, f = 0, f_sh = 0;
    int E = 0, k = 0, qtype = 0;  // E: experts the router scores
    // expert-parallel layers hold experts [e_first, e_first + n_exp) of the E; others all E
    int e_first = 0, n_exp = 0;
    bool has_shared = false, has_shared_gate = false, has_bias = false;
    float* router = nullptr;   // f32 [E + 1][d]; row E = shared-expert gate vector (zeros if absent)
    float* bias = nullptr;     // f32 [E] or null
    float* router_t = nullptr; // f32 [d][ep]: rows 0..E-1 of router transposed, zero-padded to ep = ceil(E/128)*128
    int64_t ep = 0;
    // tensor-core router (prefill): rows 0..E-1 of router scaled by 2^rs and split into
    // f16 hi/lo [E][d], with upper bounds of the row 2-norms (unscaled)
    bool router_tc = false;
    __half* router_h = nullptr;
    __half* router_l = nullptr;
    float* router_nrm = nullptr;
    int router_rs = 0;
    CUtensorMap rmap_h, rmap_l;
    PiMats gate, up, down;     // held routed experts: gate/up [n_exp][f][d], down [n_exp][d][f]
    PiMats gate_sh, up_sh, down_sh;  // shared expert (n = 1)
    PiPrefillMaps maps;              // valid when maps_ok (Q4_0, prefill-GEMM shapes)
    bool maps_ok = false;
    std::vector<void*> allocs;
};

struct pi_sparse_ffn {
    pi_ctx* ctx = nullptr;
    int64_t n_embd = 0, n_ff = 0;
    int qtype = 0;
    PiMats gate, up;           // [1][n_ff][n_embd]
    // down projection repacked neuron-major: for neuron s, the n_embd weights
    // W_down[c][s] (c = 0..n_embd-1) are contiguous.
    //   Q4_0: nib [n_ff][n_embd/2] (element c of neuron s in byte c/2, low
    //         nibble for even c); scale [n_ff/32][n_embd] f16 (the GGUF block
    //         scale of W_down row c, block s/32 — shared by 32 neurons)
    //   Q8_0: q [n_ff][n_embd] int8, same scale layout
    void* down_q = nullptr;
    __half* down_d = nullptr;
    uint8_t* mask = nullptr;  // [n_ff] token bits of the current pass, zero between passes
    int32_t* wlist = nullptr;  // [n_ff] neurons marked in the pass, in marking order
    uint32_t* wctr = nullptr;  // [2] list length, next list entry to claim (zero between passes)
    uint32_t* fbar = nullptr;  // fused pass: grid barrier {count, generation}
    uint32_t* tick = nullptr;  // fused pass: [n_ff / 32] per-range tickets (zero between passes)
    bool fused = true;         // one fused launch per pass (PI_SF_SPLIT=1 at create: three launches)
    std::vector<void*> allocs;
};

// Per-stream scratch arena (grown on demand, never shrunk).
struct PiArena {
    char* base = nullptr;
    size_t cap = 0;
};

// Optional per-kernel timing (CUDA events recorded around each launch of
// the layer path on its stream; totals read back by pi_ctx_profile_read).
struct PiProfEntry {
    std::string name;
    std::vector<cudaEvent_t> beg, end;  // one pair per launch since the last read
    double total_ms = 0;
    long launches = 0;
};

struct pi_ctx {
    int device = 0;
    bool profiling = false;
    std::deque<PiProfEntry> prof;  // deque: entries never move while a scope holds one
    int sm_count = 0;
    std::mutex mu;
    std::string last_error;
    std::unordered_map<cudaStream_t, PiArena> arenas;
    uint32_t* dev_err = nullptr;  // device error word
};

// Bump allocator over an arena; every sub-buffer is 256-byte aligned.
struct PiBump {
    char* base;
    size_t off = 0;
    template <typename T>
    T* take(size_t count) {
        off = (off + 255) & ~size_t(255);
        T* p = reinterpret_cast<T*>(base + off);
        off += count * sizeof(T);
        return p;
    }
};

int pi_set_error(pi_ctx* ctx, int code, const std::string& msg);
// Kernel timing scope: records an event pair on `st` when profiling is on.
struct PiProfScope {
    pi_ctx* ctx;
    cudaStream_t st;
    const char* name;
    PiProfEntry* e = nullptr;
    PiProfScope(pi_ctx* c, cudaStream_t s, const char* name);
    ~PiProfScope();
};
int pi_cuda_check(pi_ctx* ctx, cudaError_t e, const char* what);
// Raises fn's dynamic shared-memory limit to `bytes` on the current device (once per
// kernel and device; no-op at or below the 48 KB default).
void pi_smem_attr(const void* fn, size_t bytes);
// Returns scratch of at least `bytes` for `stream` (allocating if needed).
int pi_scratch(pi_ctx* ctx, cudaStream_t stream, size_t bytes, char** out);

// Device pointers and shapes handed to the expert kernels (decode GEMV and prefill GEMM).
struct ExpertArgs {
    // routed experts
    const void* g;
    const void* u;
    const void* dn;
    const __half* gd;
    const __half* ud;
    const __half* dd;
    // shared expert (n = 1)
    const void* gs;
    const void* us;
    const void* dns;
    const __half* gsd;
    const __half* usd;
    const __half* dsd;
    int E, d, f;  // f = routed and shared width (equal)
    const int4* items;
    const int32_t* n_items;
    const int32_t* perm;
    int n_routed;  // T*k
    // activations
    const int8_t* xq;  // Q8_0 path: quantised tokens [T][d]
    const float* xs;   // Q8_0 path: scales [T][d/32]
    const float* xf;   // Q4_0 path: f32 tokens [T][d]
    // hidden
    int8_t* hq;  // Q8_0: [slots][f]
    float* hs;   // Q8_0: [slots][f/32]
    float* hf;   // Q4_0: [slots][f]
    float* y;    // [slots][d]
    // Q8_0 prefill GEMM: h as exact f16 [slots][f] (scales in hs); the gate/up GEMM
    // gathers its slots' activation rows from xq / xs itself
    __half* h16;
    // slot -> activation row: routed slot s < n_routed reads row perm[s]; shared slot
    // n_routed + t reads row sh_row0 + t. With n_routed_dev set, n_routed is *n_routed_dev
    // (known only on the device).
    const int32_t* n_routed_dev = nullptr;
    int sh_row0 = 0;
    int n_sh = 0;  // shared-expert slots
    const int8_t* xq_sh = nullptr;  // Q8_0 GEMM: shared-expert rows from here (row t) when set
    const float* xs_sh = nullptr;
};


// Prefill expert products on tcgen05 tensor cores (pi_prefill.cu): the gate/up
// GEMM gathers each slot's token row from the token-major f16 hi/lo split
// xth/xtl [T][d] and writes SwiGLU h as f16 hi/lo hh/hl [n_slots][f]; the down
// GEMM writes a.y, over work items of <= PI_GEMM_NT slots. Returns a PI_* status.
int pi_prefill_experts(pi_ctx* ctx, const pi_moe_layer* L, const ExpertArgs& a, int64_t max_items, int64_t n_slots,
                       const __half* xth, const __half* xtl, int64_t T, __half* hh, __half* hl, cudaStream_t st);
// Builds L->maps (layer create; no-op for layers the GEMM does not take).
int pi_prefill_prepare(pi_ctx* ctx, pi_moe_layer* L);
// n_embd and expert width the prefill GEMM tiles (whole 512-row / 128-row CTA blocks)
inline bool pi_prefill_shape_ok(int64_t d, int64_t f) { return d % 512 == 0 && f % 128 == 0; }
constexpr int PI_GEMM_NT = 256;     // slots per prefill work item (Q4_0)
constexpr int PI_GEMM_NT_Q8 = 128;  // slots per prefill work item (Q8_0)
// Exact Q8_0 prefill expert products (pi_prefill_q8.cu): gate/up + SwiGLU + Q8_0 h
// into a.hq/a.hs, then down into a.y, over work items of <= PI_GEMM_NT_Q8 slots.
int pi_prefill_experts_q8(pi_ctx* ctx, const pi_moe_layer* L, const ExpertArgs& a, int64_t max_items, int64_t T,
                          int64_t n_slots, int flags, cudaStream_t st);
// Builds L->maps for a Q8_0 layer (layer create; no-op for layers the GEMM does not take).
int pi_prefill_prepare_q8(pi_ctx* ctx, pi_moe_layer* L);
bool pi_prefill_q8_shape_ok(int64_t d, int64_t f);

// Layer forward pieces (pi_moe.cu)
size_t pi_moe_scratch_bytes(const pi_moe_layer* L, int64_t T, int flags);
int pi_moe_run(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, float* out, int flags, int32_t* idx_out,
               float* gates_out, int32_t* counts_out, int32_t* offsets_out, int32_t* perm_out, char* scratch,
               cudaStream_t st);
// Internal forward flag: keep the Q8_0 activations of a routing-only run (expert parallelism).
constexpr int PI_FWD_KEEP_Q8 = 1 << 30;
// Expert-parallel stages (pi_moe.cu); buffers as documented at the C ABI.
int pi_moe_ep_route_run(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, int flags, int world,
                        int32_t* idx, float* gates, float* shscale, int8_t* xq, float* xs, int32_t* send_counts,
                        int8_t* send_xq, float* send_xs, int32_t* send_eid, int32_t* slot_row, char* scratch,
                        cudaStream_t st);
size_t pi_moe_rows_scratch_bytes(const pi_moe_layer* L, int64_t n_rows);
int pi_moe_rows_run(pi_ctx* ctx, pi_moe_layer* L, int64_t n_rows, const int8_t* xq, const float* xs,
                    const int32_t* eid, float* y, char* scratch, cudaStream_t st);
int pi_moe_ep_combine_run(pi_ctx* ctx, const pi_moe_layer* L, const float* x, int64_t T, int flags, const float* gates,
                          const float* shscale, const int32_t* slot_row, const float* y_back, const float* y_shared,
                          float* out, cudaStream_t st);
// Expert-parallel forward over NVLink peer memory (pi_ep.cu) uses these two passes:
// the home tokens' routing with their Q8_0 rows kept, and the held experts over the
// received rows (row r carries up to k local expert ids eid[r*k + j], ascending, -1 for
// none) plus the shared expert over n_home home rows. Both carve from `scratch`.
struct PiEpHome {
    int32_t* idx;
    float* gates;
    float* shscale;
    int8_t* xq;
    float* xs;
};
size_t pi_moe_ep_home_bytes(const pi_moe_layer* L, int64_t T, int flags);
int pi_moe_ep_home(pi_ctx* ctx, pi_moe_layer* L, const float* x, int64_t T, int flags, char* scratch, PiEpHome* H,
                   cudaStream_t st);
struct PiRowsOut {
    float* y;            // [slots][d]: routed slots, then the shared expert's
    int32_t* slot_of;    // [n_rows * k]
    int32_t* n_routed;   // device: routed slots (the shared expert's slot of home row t is *n_routed + t)
};
size_t pi_moe_rows_multi_bytes(const pi_moe_layer* L, int64_t n_rows, int k, int64_t n_home);
int pi_moe_rows_multi_run(pi_ctx* ctx, pi_moe_layer* L, int64_t n_rows, int k, const int8_t* xq, const float* xs,
                          const int32_t* eid, int64_t n_home, const int8_t* xq_home, const float* xs_home, int flags,
                          char* scratch, PiRowsOut* out, cudaStream_t st);
// Builds L->router_t and the tensor-core router operands from L->router (prefill router kernels).
int pi_router_prepare(pi_ctx* ctx, pi_moe_layer* L);
// Fast router logits on tensor cores (pi_prefill.cu): logits[t][e] (stride E + 1),
// e < E, from the tokens split into f16 hi/lo xh/xl [T][d]; the error against the
// reference's logits is bounded by the caller's interval arithmetic.
int pi_router_logits_tc(pi_ctx* ctx, const pi_moe_layer* L, const __half* xh, const __half* xl, int64_t T,
                        float* logits, cudaStream_t st);
// Builds the tensor maps of the tensor-core router operands (layer create).
bool pi_router_maps(pi_moe_layer* L);
// Rewrites a down-projection family into the lane-tiled order the down kernels read.
int pi_tile_down_mats(pi_ctx* ctx, PiMats* m, std::vector<void*>* allocs);
// Rewrites Q8_0 gate/up rows into the lane-tiled order k_gateup_q8 reads.
int pi_tile_gateup_mats(pi_ctx* ctx, PiMats* m, std::vector<void*>* allocs);
int pi_repack_mats(pi_ctx* ctx, PiMats* m, const void* raw, int qtype, int64_t n, int64_t rows, int64_t cols,
                   int src_on_host, std::vector<void*>* allocs);
