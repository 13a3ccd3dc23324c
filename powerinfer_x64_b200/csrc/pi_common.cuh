// Shared device helpers for the MoE / sparse-FFN kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define PI_DEV __device__ __forceinline__

// GGML type ids used at the C ABI (same numbering as ggml_type).
enum { PI_QT_F32 = 0, PI_QT_F16 = 1, PI_QT_Q4_0 = 2, PI_QT_Q8_0 = 8 };

// Device error word bits (written by kernels, read by pi_ctx_check).
enum { PI_DEVERR_INDEX = 1, PI_DEVERR_TIMEOUT = 2, PI_DEVERR_SHAPE = 4 };

// Round-to-nearest IEEE ops that the compiler may not contract into FMA:
// the reference (Rust) never fuses a*b+c, so every exact-parity kernel uses
// these instead of * and +.
PI_DEV float fmul(float a, float b) { return __fmul_rn(a, b); }
PI_DEV float fadd(float a, float b) { return __fadd_rn(a, b); }
PI_DEV float fsub(float a, float b) { return __fsub_rn(a, b); }
PI_DEV float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// Correctly rounded f32 exp: exp evaluated in f64 and rounded once to f32.
// glibc's expf (what Rust's f32::exp calls on Linux) agrees with this on all
// but ~0.008% of f32 inputs, where glibc is off by one ulp; see the design
// notes on routing ties.
PI_DEV float exp_cr(float x) { return (float)exp((double)x); }

// sigmoid as the reference writes it: 1 / (1 + exp(-g)).
PI_DEV float sigmoid_ref(float g) { return fdiv(1.0f, fadd(1.0f, exp_cr(-g))); }
// g * sigmoid(g) * u, left to right.
PI_DEV float swiglu_ref(float g, float u) { return fmul(fmul(g, sigmoid_ref(g)), u); }

PI_DEV float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Q8_0 activation quantiser (one 32-block per warp, lane i holds element i):
// amax -> d = amax/127 -> id = 1/d -> q = clamp(round(x*id)) ; scale = f16(d).
// Returns q for this lane; *scale_out receives the f16-rounded scale.
PI_DEV int8_t warp_quant_q8(float x, float* scale_out) {
    float a = fabsf(x);
    float amax = (a == a) ? a : 0.0f;  // NaN never wins `abs > amax`
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float d = fdiv(amax, 127.0f);
    float id = (d != 0.0f) ? fdiv(1.0f, d) : 0.0f;
    float r = roundf(fmul(x, id));  // half away from zero, like Rust f32::round
    int q = (r != r) ? 0 : (int)fminf(127.0f, fmaxf(-127.0f, r));
    *scale_out = __half2float(__float2half_rn(d));
    return (int8_t)q;
}

// Q8_0 quantisation of four consecutive values of a 32-block whose eight quarters sit in
// eight aligned consecutive lanes (all 32 lanes of the warp call it): returns the four
// int8 values packed little-endian, with warp_quant_q8's arithmetic per value.
PI_DEV uint32_t quad_quant_q8(const float e[4], float* scale_out) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float a = fabsf(e[j]);
        amax = fmaxf(amax, (a == a) ? a : 0.0f);  // NaN never wins `abs > amax`
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = fdiv(amax, 127.0f);
    const float id = (d != 0.0f) ? fdiv(1.0f, d) : 0.0f;
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float r = roundf(fmul(e[j], id));  // half away from zero, like Rust f32::round
        const int q = (r != r) ? 0 : (int)fminf(127.0f, fmaxf(-127.0f, r));
        packed |= (uint32_t)(q & 0xff) << (8 * j);
    }
    *scale_out = __half2float(__float2half_rn(d));
    return packed;
}

PI_DEV int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

PI_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Streaming 16-byte load that does not pollute L1 (weights are read once).
// Programmatic dependent launch (kernels launched with pi_pdl_launch): pdl_wait blocks
// until the stream's previous kernel has completed and its writes are visible (a no-op
// for a normal launch); pdl_trigger lets the next kernel start launching once every CTA
// of this one has run it. Every CTA calls pdl_wait unconditionally, before it can return
// and before it touches anything the previous kernel writes (reads of constant weights may
// come first), so that a kernel never completes before the one it follows.
PI_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
PI_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

PI_DEV int4 ld_stream(const void* p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

#ifdef __CUDACC__
// Launch with programmatic stream serialisation (the kernel must start with pdl_wait()).
template <typename... KArgs, typename... Args>
inline void pi_pdl_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}
#endif
