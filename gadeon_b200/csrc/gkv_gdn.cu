// gkv_gdn.cu -- rollback of the Gated-DeltaNet layers' state after an
// accepted speculative prefix: the step that runs beside the KV truncate in
// every MTP cycle (leok7v/gadeon Engine.decodeSpecStep ->
// rollbackGDN, LLM/src/CoreML/Engine.swift:2678-2716).
//
//   mtp_rollback_kernel  MtpRollback.stateAfter (LLM/src/CoreML/MtpRollback.swift
//                        :20-60): S_m = exp(g[m-1]) S0 + sum_{t<m}
//                        exp(g[m-1]-g[t]) outer(k_t, delta_t), per value head.
//   conv_rollback_kernel Engine.convFromProj (Engine.swift:2719-2740): the
//                        conv tail after m committed tokens.
//
// Both are HBM-bound streams (the recurrent state is read and written once);
// items are (sequence, GDN layer) pairs of a batch, each with its own m.
// The per-item m travels in the kernel parameters, so a call allocates
// nothing and needs no upload.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <utility>

#include <cmath>
#include <cstdarg>
#include <cstdio>

#include "gadeon_kv.h"
#include "gkv_kernels.cuh"

namespace gkv {
namespace {

constexpr int kMaxItemsPerLaunch = 2048;
constexpr int kMaxChunk = 64;  // verify width C

// State storage T: float (fp32 in and out) or __half -- the reference's own
// storage (Engine.rollbackGDN reads the fp16 gdnState arrays, rebuilds in
// fp32 and writes them back through fp16Array, Engine.swift:2697-2705):
// widened exactly on load, rounded to nearest even on store, the fp32
// arithmetic in between unchanged.
template <typename T>
struct RollbackParams {
    int32_t H, DK, DV, C;
    const T *s0;
    const float *delta, *k, *gcum;
    T *out;
    int32_t m[kMaxItemsPerLaunch];
};

template <typename T>
struct ConvParams {
    int32_t CD, taps, C;
    const float *proj;
    const T *pre;
    T *out;
    int32_t m[kMaxItemsPerLaunch];
};

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// COLS consecutive fp16 state elements moved as one 16-byte access.
template <typename T, int COLS>
struct Cols;
__device__ __forceinline__ float2 h2_to_f2(uint32_t x) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&x));
}
__device__ __forceinline__ uint32_t f2_to_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
template <>
struct Cols<__half, 8> {
    using raw = uint4;
    __device__ static void unpack(const raw &r, float (&v)[8]) {
        const float2 a = h2_to_f2(r.x), b = h2_to_f2(r.y), c = h2_to_f2(r.z), d = h2_to_f2(r.w);
        v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y, v[4] = c.x, v[5] = c.y, v[6] = d.x, v[7] = d.y;
    }
    __device__ static raw pack(const float (&v)[8]) {
        return make_uint4(f2_to_h2(v[0], v[1]), f2_to_h2(v[2], v[3]), f2_to_h2(v[4], v[5]), f2_to_h2(v[6], v[7]));
    }
};

// One CTA per (item, value head): the head's [DK, DV] state streams through
// in float4s, kUnroll of them in flight per thread; the m gate weights are
// computed once per CTA and the head's k / delta rows stay in L1.
constexpr int kRollThreads = 256;
constexpr int kUnroll = 4;

__device__ __forceinline__ float4 rollback_elem(const RollbackParams<float> &p, const float *w, float eM,
                                                const float *kk, const float *dd, int m, int e4, float4 s) {
    const int i = e4 * 4 / p.DV, j = e4 * 4 % p.DV;
    // reference order: out = eM * s0, then out += (w_t * k_t[i]) * delta_t[j]
    // for t ascending, each multiply and add rounded on its own
    float4 o = make_float4(__fmul_rn(eM, s.x), __fmul_rn(eM, s.y), __fmul_rn(eM, s.z), __fmul_rn(eM, s.w));
    for (int t = 0; t < m; ++t) {
        const float wk = __fmul_rn(w[t], __ldg(kk + t * p.DK + i));
        const float4 d = __ldg(reinterpret_cast<const float4 *>(dd + t * p.DV + j));
        o.x = __fadd_rn(o.x, __fmul_rn(wk, d.x));
        o.y = __fadd_rn(o.y, __fmul_rn(wk, d.y));
        o.z = __fadd_rn(o.z, __fmul_rn(wk, d.z));
        o.w = __fadd_rn(o.w, __fmul_rn(wk, d.w));
    }
    return o;
}

// Any DV: one element per thread step, same operation order as the vector
// path.
template <typename T>
__device__ __forceinline__ float rollback_scalar(const RollbackParams<T> &p, const float *w, float eM,
                                                 const float *kk, const float *dd, int m, int e, float s) {
    const int i = e / p.DV, j = e % p.DV;
    float o = __fmul_rn(eM, s);
    for (int t = 0; t < m; ++t)
        o = __fadd_rn(o, __fmul_rn(__fmul_rn(w[t], __ldg(kk + t * p.DK + i)), __ldg(dd + t * p.DV + j)));
    return o;
}

// VEC (fp32 only): float4 rows; otherwise one element at a time.
template <typename T, bool VEC>
__global__ void __launch_bounds__(kRollThreads) mtp_rollback_kernel(const __grid_constant__ RollbackParams<T> p) {
    __shared__ float w[kMaxChunk];
    __shared__ float eM;
    const int hs = blockIdx.x;  // item * H + head
    const int m = p.m[hs / p.H];
    const float *g = p.gcum + (int64_t)hs * p.C;
    if (threadIdx.x < m) w[threadIdx.x] = expf(g[m - 1] - g[threadIdx.x]);
    if (threadIdx.x == 0) eM = expf(g[m - 1]);
    __syncthreads();
    const int64_t sbase = (int64_t)hs * p.DK * p.DV;
    const float *kk = p.k + (int64_t)hs * p.C * p.DK;
    const float *dd = p.delta + (int64_t)hs * p.C * p.DV;
    const float e = eM;
    if constexpr (VEC) {
        static_assert(sizeof(T) == 4, "float4 rows of an fp32 state");
        const int nv4 = p.DK * p.DV / 4;
        const float4 *s4 = reinterpret_cast<const float4 *>(p.s0 + sbase);
        float4 *o4 = reinterpret_cast<float4 *>(p.out + sbase);
        for (int base = threadIdx.x; base < nv4; base += kUnroll * kRollThreads) {
            float4 s[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int e4 = base + u * kRollThreads;
                if (e4 < nv4) s[u] = __ldcs(s4 + e4);
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int e4 = base + u * kRollThreads;
                if (e4 < nv4) __stcs(o4 + e4, rollback_elem(p, w, e, kk, dd, m, e4, s[u]));
            }
        }
    } else {
        const int n = p.DK * p.DV;
        for (int x = threadIdx.x; x < n; x += kRollThreads)
            p.out[sbase + x] = from_f32<T>(rollback_scalar(p, w, e, kk, dd, m, x, to_f32(p.s0[sbase + x])));
    }
}

// grid (ceil(CD / 256), items): thread = one channel c of one item, all its
// taps; reads of proj rows and writes of the [CD, taps] tail are coalesced
// across the warp's consecutive channels.  fp16 storage: a proj value is
// rounded to nearest even (Float16(val), Engine.swift:2733), a carried tap
// is copied as it was.
template <typename T>
__global__ void __launch_bounds__(256) conv_rollback_kernel(const __grid_constant__ ConvParams<T> p) {
    const int item = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= p.CD) return;
    const int m = p.m[item];
    const float *proj = p.proj + (int64_t)item * p.C * p.CD + c;
    const int64_t tail = ((int64_t)item * p.CD + c) * p.taps;
    for (int t = 0; t < p.taps; ++t) {
        const int pos = m - p.taps + t;
        p.out[tail + t] = pos >= 0 ? from_f32<T>(__ldcs(proj + (int64_t)pos * p.CD)) : p.pre[tail + m + t];
    }
}

// Vector form for conv_dim % 8 == 0, taps <= 4 and 16-byte aligned arrays:
// thread = 8 consecutive channels of one item with all their taps, so its
// slice of the [CD, taps] tail is 8*TAPS contiguous elements (a multiple of
// 16 bytes for fp16 and fp32) moved with 16-byte loads and stores; the proj
// row slices are two float4 loads per tap.  Same values as the scalar kernel.
constexpr int kConvVecThreads = 128;

// Element e of a slice kept as 32-bit words in registers (compile-time e):
// fp32 one element per word, fp16 two (raw bits, so carried taps are copied
// exactly).
template <typename T>
struct Words {
    static constexpr int PER = 4 / (int)sizeof(T);
    __device__ __forceinline__ static uint32_t get(const uint32_t *w, int e) {
        return PER == 1 ? w[e] : (w[e >> 1] >> (16 * (e & 1))) & 0xffffu;
    }
    __device__ __forceinline__ static void set(uint32_t *w, int e, uint32_t bits) {
        if (PER == 1)
            w[e] = bits;
        else if (e & 1)
            w[e >> 1] = (w[e >> 1] & 0x0000ffffu) | (bits << 16);
        else
            w[e >> 1] = (w[e >> 1] & 0xffff0000u) | bits;
    }
    __device__ __forceinline__ static uint32_t bits_of(float x) {
        if (PER == 1) return __float_as_uint(x);
        return (uint32_t)__half_as_ushort(__float2half_rn(x));
    }
};

// One thread's slice for an accepted length m with KEEP = max(TAPS - m, 0)
// carried taps: out tap t < KEEP is carried tap t + (TAPS - KEEP) = m + t of
// pre; out tap t >= KEEP is projection row m - TAPS + t (>= 0).
template <typename T, int TAPS, int KEEP>
__device__ __forceinline__ void conv_slice(const ConvParams<T> &p, int item, int c0, int64_t tail, int m) {
    using W = Words<T>;
    constexpr int NW = 8 * TAPS / W::PER;
    uint32_t pre[NW], out[NW];
    if constexpr (KEEP > 0) {
        const uint4 *src = reinterpret_cast<const uint4 *>(p.pre + tail);
#pragma unroll
        for (int v = 0; v < NW / 4; ++v) {
            const uint4 x = __ldcs(src + v);
            pre[4 * v] = x.x, pre[4 * v + 1] = x.y, pre[4 * v + 2] = x.z, pre[4 * v + 3] = x.w;
        }
    }
#pragma unroll
    for (int w = 0; w < NW; ++w) out[w] = 0u;
#pragma unroll
    for (int t = 0; t < TAPS; ++t) {
        if (t < KEEP) {
#pragma unroll
            for (int c = 0; c < 8; ++c) W::set(out, c * TAPS + t, W::get(pre, c * TAPS + t + (TAPS - KEEP)));
        } else {
            const float4 *row =
                reinterpret_cast<const float4 *>(p.proj + ((int64_t)item * p.C + (m - TAPS + t)) * p.CD + c0);
            const float4 a = __ldcs(row), b = __ldcs(row + 1);
            const float r[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int c = 0; c < 8; ++c) W::set(out, c * TAPS + t, W::bits_of(r[c]));
        }
    }
    uint4 *dst = reinterpret_cast<uint4 *>(p.out + tail);
#pragma unroll
    for (int v = 0; v < NW / 4; ++v) __stcs(dst + v, make_uint4(out[4 * v], out[4 * v + 1], out[4 * v + 2], out[4 * v + 3]));
}

template <typename T, int TAPS, int THREADS = kConvVecThreads>
__device__ __forceinline__ void conv_vec_block(const ConvParams<T> &p, int item, int bx) {
    static_assert((8 * TAPS / Words<T>::PER) % 4 == 0, "whole 16-byte vectors");
    const int c0 = (bx * THREADS + threadIdx.x) * 8;
    if (c0 >= p.CD) return;
    const int m = p.m[item];
    const int64_t tail = ((int64_t)item * p.CD + c0) * TAPS;
    switch (m >= TAPS ? 0 : TAPS - m) {  // carried taps kept
        case 0: conv_slice<T, TAPS, 0>(p, item, c0, tail, m); break;
        case 1: if constexpr (TAPS > 1) conv_slice<T, TAPS, 1>(p, item, c0, tail, m); break;
        case 2: if constexpr (TAPS > 2) conv_slice<T, TAPS, 2>(p, item, c0, tail, m); break;
        case 3: if constexpr (TAPS > 3) conv_slice<T, TAPS, 3>(p, item, c0, tail, m); break;
        default: break;
    }
}

// grid (ceil(CD / 8 / 128), items)
template <typename T, int TAPS>
__global__ void __launch_bounds__(kConvVecThreads) conv_rollback_vec_kernel(const __grid_constant__ ConvParams<T> p) {
    conv_vec_block<T, TAPS>(p, blockIdx.y, blockIdx.x);
}

// Fast path for the verify widths MTP uses (C <= kFastC), DV a multiple of
// COLS with DV <= COLS * kRollThreads, DK <= kFastDK: thread = one group cg
// of COLS state columns and rows r0, r0 + rstride, ...; its delta_t[cg] for
// t < m live in registers, the m rows of w_t * k_t (the reference's wk) in
// shared memory, read as warp-wide broadcasts when a warp covers one row.
// The state streams through UNROLL 16-byte loads in flight per thread; the
// first batch is issued before the prologue so its latency overlaps it.
constexpr int kFastC = 8;
constexpr int kFastDK = 256;
constexpr int kFastUnroll = 4;  // fp32: 8 needs 80 registers, 3 CTAs/SM and 0.89 of the HBM copy rate; 4 reaches 0.94
// fp16 state kernel shape, measured on config 6 (128 sequences x 3 GDN layers,
// 32 heads of 128 x 128, C = 5): state launch 0.164 ms with 128 threads x 8
// columns x 4 loads in flight (74 registers); 256 threads: 0.206 ms; 8 loads:
// 0.178 ms; 4 columns x 8 loads: 0.186 ms; 64 threads: 0.162 ms.  Smaller CTAs
// win because each pays a fixed prologue (gate weights, wk rows, delta) on
// half the bytes an fp32 CTA streams.
constexpr int kF16Cols = 8;       // fp16 columns per thread (one 16-byte access)
constexpr int kF16Unroll = 4;     // state loads in flight per thread
constexpr int kF16Threads = 128;
constexpr int kF16NarrowC = 5;              // verify width of the MTP cycle (token + 4 drafts)

// fp32 state: thread = one float4 column group (64 registers, 4 CTAs/SM).
__device__ __forceinline__ void state_fast_f32_block(const RollbackParams<float> &p, int hs) {
    __shared__ float kw[kFastC][kFastDK];
    __shared__ float eM_s;
    const int m = p.m[hs / p.H];
    const int ncg = p.DV >> 2;
    const int rstride = kRollThreads / ncg;
    const int cg = threadIdx.x % ncg, r0 = threadIdx.x / ncg;
    const bool active = r0 < rstride;
    const int64_t sbase = (int64_t)hs * p.DK * p.DV;
    const float4 *s4 = reinterpret_cast<const float4 *>(p.s0 + sbase);
    float4 *o4 = reinterpret_cast<float4 *>(p.out + sbase);
    float4 s[kFastUnroll];
#pragma unroll
    for (int u = 0; u < kFastUnroll; ++u) {
        const int i = r0 + u * rstride;
        if (active && i < p.DK) s[u] = __ldcs(s4 + (int64_t)i * ncg + cg);
    }
    // prologue: gate weights, wk rows, this thread's delta column
    const float *g = p.gcum + (int64_t)hs * p.C;
    const float gLast = g[m - 1];
    const float *kk = p.k + (int64_t)hs * p.C * p.DK;
    for (int x = threadIdx.x; x < m * p.DK; x += kRollThreads) {
        const int t = x / p.DK, i = x - t * p.DK;
        kw[t][i] = __fmul_rn(expf(gLast - g[t]), kk[x]);
    }
    if (threadIdx.x == 0) eM_s = expf(gLast);
    float4 d[kFastC];
    const float4 *d4 = reinterpret_cast<const float4 *>(p.delta + (int64_t)hs * p.C * p.DV);
#pragma unroll
    for (int t = 0; t < kFastC; ++t)
        if (t < m) d[t] = __ldg(d4 + t * ncg + cg);
    __syncthreads();
    if (!active) return;
    const float eM = eM_s;
    for (int base = r0;; base += kFastUnroll * rstride) {
#pragma unroll
        for (int u = 0; u < kFastUnroll; ++u) {
            const int i = base + u * rstride;
            if (i < p.DK) {
                float4 o = make_float4(__fmul_rn(eM, s[u].x), __fmul_rn(eM, s[u].y), __fmul_rn(eM, s[u].z),
                                       __fmul_rn(eM, s[u].w));
#pragma unroll
                for (int t = 0; t < kFastC; ++t) {
                    if (t < m) {
                        const float wk = kw[t][i];
                        o.x = __fadd_rn(o.x, __fmul_rn(wk, d[t].x));
                        o.y = __fadd_rn(o.y, __fmul_rn(wk, d[t].y));
                        o.z = __fadd_rn(o.z, __fmul_rn(wk, d[t].z));
                        o.w = __fadd_rn(o.w, __fmul_rn(wk, d[t].w));
                    }
                }
                __stcs(o4 + (int64_t)i * ncg + cg, o);
            }
        }
        const int next = base + kFastUnroll * rstride;
        if (next >= p.DK) break;
#pragma unroll
        for (int u = 0; u < kFastUnroll; ++u) {
            const int i = next + u * rstride;
            if (i < p.DK) s[u] = __ldcs(s4 + (int64_t)i * ncg + cg);
        }
    }
}

__global__ void __launch_bounds__(kRollThreads) mtp_rollback_fast_f32_kernel(const __grid_constant__ RollbackParams<float> p) {
    state_fast_f32_block(p, blockIdx.x);
}

// The stream loop of the fp16 kernel for a compile-time accepted length M:
// rows r0, r0 + rstride, ... of the head, UNROLL loads in flight (the first
// batch already loaded into s), out = eM*s then += wk_t*delta_t, t < M.
template <typename V, typename R, int COLS, int UNROLL, int MAXC, int M>
__device__ __forceinline__ void roll_rows(int DK, int r0, int rstride, int ncg, int cg, float eM,
                                          const float (&kw)[kFastC][kFastDK], const float (&d)[MAXC][COLS],
                                          R (&s)[UNROLL], const R *s4, R *o4) {
    for (int base = r0;; base += UNROLL * rstride) {
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int i = base + u * rstride;
            if (i < DK) {
                float o[COLS];
                V::unpack(s[u], o);
#pragma unroll
                for (int c = 0; c < COLS; ++c) o[c] = __fmul_rn(eM, o[c]);
#pragma unroll
                for (int t = 0; t < M; ++t) {
                    const float wk = kw[t][i];
#pragma unroll
                    for (int c = 0; c < COLS; ++c) o[c] = __fadd_rn(o[c], __fmul_rn(wk, d[t][c]));
                }
                __stcs(o4 + (int64_t)i * ncg + cg, V::pack(o));
            }
        }
        const int next = base + UNROLL * rstride;
        if (next >= DK) break;
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int i = next + u * rstride;
            if (i < DK) s[u] = __ldcs(s4 + (int64_t)i * ncg + cg);
        }
    }
}

// fp16 state: thread = COLS columns moved as one 8- or 16-byte access, the
// same arithmetic per element as the fp32 kernel.
template <typename T, int COLS, int UNROLL, int MAXC, int THREADS>
__device__ __forceinline__ void state_fast_block(const RollbackParams<T> &p, int hs) {
    using V = Cols<T, COLS>;
    using R = typename V::raw;
    __shared__ float kw[kFastC][kFastDK];
    __shared__ float eM_s;
    const int m = p.m[hs / p.H];
    const int ncg = p.DV / COLS;
    const int rstride = THREADS / ncg;
    const int cg = threadIdx.x % ncg, r0 = threadIdx.x / ncg;
    const bool active = r0 < rstride;
    const int64_t sbase = (int64_t)hs * p.DK * p.DV;
    const R *s4 = reinterpret_cast<const R *>(p.s0 + sbase);
    R *o4 = reinterpret_cast<R *>(p.out + sbase);
    R s[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        const int i = r0 + u * rstride;
        if (active && i < p.DK) s[u] = __ldcs(s4 + (int64_t)i * ncg + cg);
    }
    // prologue: gate weights, wk rows, this thread's delta columns
    const float *g = p.gcum + (int64_t)hs * p.C;
    const float gLast = g[m - 1];
    const float *kk = p.k + (int64_t)hs * p.C * p.DK;
    for (int x = threadIdx.x; x < m * p.DK; x += THREADS) {
        const int t = x / p.DK, i = x - t * p.DK;
        kw[t][i] = __fmul_rn(expf(gLast - g[t]), kk[x]);
    }
    if (threadIdx.x == 0) eM_s = expf(gLast);
    float d[MAXC][COLS];
    const float4 *d4 = reinterpret_cast<const float4 *>(p.delta + (int64_t)hs * p.C * p.DV);
#pragma unroll
    for (int t = 0; t < MAXC; ++t)
        if (t < m) {
#pragma unroll
            for (int q = 0; q < COLS / 4; ++q) {
                const float4 x = __ldg(d4 + (t * ncg + cg) * (COLS / 4) + q);
                d[t][4 * q] = x.x, d[t][4 * q + 1] = x.y, d[t][4 * q + 2] = x.z, d[t][4 * q + 3] = x.w;
            }
        }
    __syncthreads();
    if (!active) return;
    const float eM = eM_s;
    // m is the same for the whole CTA: a copy of the stream loop per m issues
    // exactly m multiply-add steps per element instead of MAXC guarded ones
    switch (m) {
#define GKV_ROLL_CASE(M) \
    case M:              \
        if constexpr (M <= MAXC) roll_rows<V, R, COLS, UNROLL, MAXC, M>(p.DK, r0, rstride, ncg, cg, eM, kw, d, s, s4, o4); \
        break;
        GKV_ROLL_CASE(1)
        GKV_ROLL_CASE(2)
        GKV_ROLL_CASE(3)
        GKV_ROLL_CASE(4)
        GKV_ROLL_CASE(5)
        GKV_ROLL_CASE(6)
        GKV_ROLL_CASE(7)
        GKV_ROLL_CASE(8)
#undef GKV_ROLL_CASE
        default:
            break;
    }
}

template <typename T, int COLS, int UNROLL, int MAXC, int THREADS>
__global__ void __launch_bounds__(THREADS) mtp_rollback_fast_kernel(const __grid_constant__ RollbackParams<T> p) {
    state_fast_block<T, COLS, UNROLL, MAXC, THREADS>(p, blockIdx.x);
}

// The whole of Engine.rollbackGDN for a batch in one launch (fp16 storage):
// blocks [0, state_blocks) roll back one (item, value head) state each,
// the rest one 1,024-channel slice of an item's conv tail each.  The two
// parts touch disjoint memory, so the conv blocks, dispatched last, fill the
// state stream's tail instead of running as a launch of their own.
template <typename T>
struct GdnParams {
    RollbackParams<T> s;
    ConvParams<T> c;
    int32_t state_blocks, conv_bx;
};

template <int MAXC, int TAPS>
__global__ void __launch_bounds__(kF16Threads) gdn_rollback_f16_kernel(const __grid_constant__ GdnParams<__half> p) {
    if ((int)blockIdx.x < p.state_blocks) {
        state_fast_block<__half, kF16Cols, kF16Unroll, MAXC, kF16Threads>(p.s, blockIdx.x);
    } else {
        const int b = (int)blockIdx.x - p.state_blocks;
        conv_vec_block<__half, TAPS, kF16Threads>(p.c, b / p.conv_bx, b % p.conv_bx);
    }
}

// fp32 storage: 256-thread blocks, the fp32 state body, conv slices of 2,048
// channels.
template <int TAPS>
__global__ void __launch_bounds__(kRollThreads) gdn_rollback_f32_kernel(const __grid_constant__ GdnParams<float> p) {
    if ((int)blockIdx.x < p.state_blocks) {
        state_fast_f32_block(p.s, blockIdx.x);
    } else {
        const int b = (int)blockIdx.x - p.state_blocks;
        conv_vec_block<float, TAPS, kRollThreads>(p.c, b / p.conv_bx, b % p.conv_bx);
    }
}

bool misaligned(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) != 0; }

// Argument checks of the state rollback; on success *fast tells whether
// the 16-byte-column kernel applies (else the element-wise one).
template <typename T>
int check_state_args(int32_t n_items, const int32_t *m, int32_t H, int32_t DK, int32_t DV, int32_t C,
                     const T *s0, const float *delta, const float *k, const float *gcum, const T *out, bool *vec_out,
                     bool *fast_out) {
    constexpr bool F16 = sizeof(T) == 2;
    if (n_items < 0 || H < 1 || DK < 1 || DV < 1 || C < 1)
        return report_error(GKV_ERR_INVALID, "n_items=%d H=%d DK=%d DV=%d C=%d", n_items, H, DK, DV, C);
    if (C > kMaxChunk) return report_error(GKV_ERR_UNSUPPORTED, "C=%d > %d", C, kMaxChunk);
    if (H > (1 << 20)) return report_error(GKV_ERR_CAPACITY, "H=%d", H);
    if ((int64_t)DK * DV > (1LL << 30)) return report_error(GKV_ERR_CAPACITY, "DK*DV=%lld", (long long)DK * DV);
    if (n_items == 0) return GKV_OK;
    if (!m || !s0 || !delta || !k || !gcum || !out) return report_error(GKV_ERR_INVALID, "null pointer");
    for (const auto &b : {std::make_pair((const void *)s0, "s0"), std::make_pair((const void *)delta, "delta"),
                          std::make_pair((const void *)k, "k"), std::make_pair((const void *)gcum, "gcum"),
                          std::make_pair((const void *)out, "out")})
        if (const int rc = check_reachable(b.first, -1, false, b.second)) return rc;
    if ((reinterpret_cast<uintptr_t>(delta) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(gcum)) & 3)
        return report_error(GKV_ERR_INVALID, "fp32 arrays must be 4-byte aligned");
    if ((reinterpret_cast<uintptr_t>(s0) | reinterpret_cast<uintptr_t>(out)) & (sizeof(T) - 1))
        return report_error(GKV_ERR_INVALID, "state arrays must be %d-byte aligned", (int)sizeof(T));
    // 16-byte rows: fp32 as float4 (DV % 4 == 0), fp16 as 8 halves (DV % 8 == 0)
    constexpr int COLS = F16 ? kF16Cols : 4;
    const bool vec = DV % COLS == 0 && !misaligned(s0) && !misaligned(delta) && !misaligned(out);
    const bool fast = vec && C <= kFastC && DK <= kFastDK && DV <= COLS * (F16 ? kF16Threads : kRollThreads);
    for (int32_t i = 0; i < n_items; ++i)
        if (m[i] < 1 || m[i] > C) return report_error(GKV_ERR_INVALID, "m[%d]=%d outside 1..%d", i, m[i], C);
    *vec_out = vec;
    *fast_out = fast;
    return GKV_OK;
}

template <typename T>
void fill_state_params(RollbackParams<T> &p, int32_t first, int32_t cnt, const int32_t *m, int32_t H, int32_t DK,
                       int32_t DV, int32_t C, const T *s0, const float *delta, const float *k, const float *gcum,
                       T *out) {
    p.H = H;
    p.DK = DK;
    p.DV = DV;
    p.C = C;
    const int64_t hs0 = (int64_t)first * H;
    p.s0 = s0 + hs0 * DK * DV;
    p.delta = delta + hs0 * C * DV;
    p.k = k + hs0 * C * DK;
    p.gcum = gcum + hs0 * C;
    p.out = out + hs0 * DK * DV;
    for (int32_t i = 0; i < cnt; ++i) p.m[i] = m[first + i];
}

template <typename T>
int mtp_rollback_impl(int32_t n_items, const int32_t *m, int32_t H, int32_t DK, int32_t DV, int32_t C,
                      const T *s0, const float *delta, const float *k, const float *gcum, T *out, void *stream) {
    constexpr bool F16 = sizeof(T) == 2;
    constexpr int COLS = F16 ? kF16Cols : 4;
    bool vec = false, fast = false;
    if (const int rc = check_state_args<T>(n_items, m, H, DK, DV, C, s0, delta, k, gcum, out, &vec, &fast)) return rc;
    if (n_items == 0) return GKV_OK;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // items per launch: what the parameter block's m[] holds
    const int32_t per = kMaxItemsPerLaunch;
    for (int32_t first = 0; first < n_items; first += per) {
        const int32_t cnt = n_items - first < per ? n_items - first : per;
        RollbackParams<T> p{};
        fill_state_params<T>(p, first, cnt, m, H, DK, DV, C, s0, delta, k, gcum, out);
        const unsigned blocks = (unsigned)((int64_t)cnt * H);
        if constexpr (!F16) {
            if (fast)
                mtp_rollback_fast_f32_kernel<<<blocks, kRollThreads, 0, st>>>(p);
            else if (vec)
                mtp_rollback_kernel<T, true><<<blocks, kRollThreads, 0, st>>>(p);
            else
                mtp_rollback_kernel<T, false><<<blocks, kRollThreads, 0, st>>>(p);
        } else {
            if (fast && C <= kF16NarrowC)
                mtp_rollback_fast_kernel<T, COLS, kF16Unroll, kF16NarrowC, kF16Threads>
                    <<<blocks, kF16Threads, 0, st>>>(p);
            else if (fast)
                mtp_rollback_fast_kernel<T, COLS, kF16Unroll, kFastC, kF16Threads><<<blocks, kF16Threads, 0, st>>>(p);
            else
                mtp_rollback_kernel<T, false><<<blocks, kRollThreads, 0, st>>>(p);
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return report_error(GKV_ERR_CUDA, "mtp_rollback launch: %s", cudaGetErrorString(e));
    }
    return GKV_OK;
}

template <typename T>
int check_conv_args(int32_t n_items, const int32_t *m, int32_t conv_dim, int32_t taps, int32_t C, const float *proj,
                    const T *pre, const T *out, bool *vec_out) {
    if (n_items < 0 || conv_dim < 1 || taps < 1 || C < 1)
        return report_error(GKV_ERR_INVALID, "n_items=%d conv_dim=%d taps=%d C=%d", n_items, conv_dim, taps, C);
    if (n_items == 0) return GKV_OK;
    if (!m || !proj || !pre || !out) return report_error(GKV_ERR_INVALID, "null pointer");
    for (const auto &b : {std::make_pair((const void *)proj, "proj"), std::make_pair((const void *)pre, "pre"),
                          std::make_pair((const void *)out, "out")})
        if (const int rc = check_reachable(b.first, -1, false, b.second)) return rc;
    if ((reinterpret_cast<uintptr_t>(proj) & 3) ||
        ((reinterpret_cast<uintptr_t>(pre) | reinterpret_cast<uintptr_t>(out)) & (sizeof(T) - 1)))
        return report_error(GKV_ERR_INVALID, "proj must be 4-byte aligned, pre/out %d-byte", (int)sizeof(T));
    for (int32_t i = 0; i < n_items; ++i)
        if (m[i] < 1 || m[i] > C) return report_error(GKV_ERR_INVALID, "m[%d]=%d outside 1..%d", i, m[i], C);
    *vec_out = conv_dim % 8 == 0 && taps <= 4 && !misaligned(proj) && !misaligned(pre) && !misaligned(out);
    return GKV_OK;
}

template <typename T>
void fill_conv_params(ConvParams<T> &p, int32_t first, int32_t cnt, const int32_t *m, int32_t conv_dim, int32_t taps,
                      int32_t C, const float *proj, const T *pre, T *out) {
    p.CD = conv_dim;
    p.taps = taps;
    p.C = C;
    p.proj = proj + (int64_t)first * C * conv_dim;
    p.pre = pre + (int64_t)first * conv_dim * taps;
    p.out = out + (int64_t)first * conv_dim * taps;
    for (int32_t i = 0; i < cnt; ++i) p.m[i] = m[first + i];
}

template <typename T>
int conv_rollback_impl(int32_t n_items, const int32_t *m, int32_t conv_dim, int32_t taps, int32_t C,
                       const float *proj, const T *pre, T *out, void *stream) {
    bool vec = false;
    if (const int rc = check_conv_args<T>(n_items, m, conv_dim, taps, C, proj, pre, out, &vec)) return rc;
    if (n_items == 0) return GKV_OK;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int32_t first = 0; first < n_items; first += kMaxItemsPerLaunch) {
        const int32_t cnt = n_items - first < kMaxItemsPerLaunch ? n_items - first : kMaxItemsPerLaunch;
        ConvParams<T> p{};
        fill_conv_params<T>(p, first, cnt, m, conv_dim, taps, C, proj, pre, out);
        if (vec) {
            const dim3 vgrid((unsigned)((conv_dim / 8 + kConvVecThreads - 1) / kConvVecThreads), (unsigned)cnt);
            switch (taps) {
                case 1: conv_rollback_vec_kernel<T, 1><<<vgrid, kConvVecThreads, 0, st>>>(p); break;
                case 2: conv_rollback_vec_kernel<T, 2><<<vgrid, kConvVecThreads, 0, st>>>(p); break;
                case 3: conv_rollback_vec_kernel<T, 3><<<vgrid, kConvVecThreads, 0, st>>>(p); break;
                default: conv_rollback_vec_kernel<T, 4><<<vgrid, kConvVecThreads, 0, st>>>(p); break;
            }
        } else {
            const dim3 grid((unsigned)((conv_dim + 255) / 256), (unsigned)cnt);
            conv_rollback_kernel<T><<<grid, 256, 0, st>>>(p);
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return report_error(GKV_ERR_CUDA, "conv_rollback launch: %s", cudaGetErrorString(e));
    }
    return GKV_OK;
}

// State and conv tail of every item in one launch when both take their
// vector kernels; otherwise the two launches of the separate entry points.
template <typename T>
int gdn_rollback_impl(int32_t n_items, const int32_t *m, int32_t H, int32_t DK, int32_t DV, int32_t C, const T *s0,
                      const float *delta, const float *k, const float *gcum, T *s_out, int32_t conv_dim,
                      int32_t taps, const float *proj, const T *pre, T *conv_out, void *stream) {
    constexpr bool F16 = sizeof(T) == 2;
    constexpr int THREADS = F16 ? kF16Threads : kRollThreads;  // the state kernel's block size
    bool svec = false, sfast = false, cvec = false;
    if (const int rc = check_state_args<T>(n_items, m, H, DK, DV, C, s0, delta, k, gcum, s_out, &svec, &sfast))
        return rc;
    if (const int rc = check_conv_args<T>(n_items, m, conv_dim, taps, C, proj, pre, conv_out, &cvec)) return rc;
    if (n_items == 0) return GKV_OK;
    if (!sfast || !cvec) {
        if (const int rc = mtp_rollback_impl<T>(n_items, m, H, DK, DV, C, s0, delta, k, gcum, s_out, stream))
            return rc;
        return conv_rollback_impl<T>(n_items, m, conv_dim, taps, C, proj, pre, conv_out, stream);
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int32_t conv_bx = (conv_dim / 8 + THREADS - 1) / THREADS;
    const bool narrow = C <= kF16NarrowC;
    for (int32_t first = 0; first < n_items; first += kMaxItemsPerLaunch) {
        const int32_t cnt = n_items - first < kMaxItemsPerLaunch ? n_items - first : kMaxItemsPerLaunch;
        GdnParams<T> p{};
        fill_state_params<T>(p.s, first, cnt, m, H, DK, DV, C, s0, delta, k, gcum, s_out);
        fill_conv_params<T>(p.c, first, cnt, m, conv_dim, taps, C, proj, pre, conv_out);
        p.state_blocks = cnt * H;
        p.conv_bx = conv_bx;
        const unsigned blocks = (unsigned)((int64_t)cnt * H + (int64_t)cnt * conv_bx);
        if constexpr (F16) {
#define GKV_GDN_LAUNCH(MAXC)                                                                                \
    switch (taps) {                                                                                         \
        case 1: gdn_rollback_f16_kernel<MAXC, 1><<<blocks, kF16Threads, 0, st>>>(p); break;                 \
        case 2: gdn_rollback_f16_kernel<MAXC, 2><<<blocks, kF16Threads, 0, st>>>(p); break;                 \
        case 3: gdn_rollback_f16_kernel<MAXC, 3><<<blocks, kF16Threads, 0, st>>>(p); break;                 \
        default: gdn_rollback_f16_kernel<MAXC, 4><<<blocks, kF16Threads, 0, st>>>(p); break;                \
    }
            if (narrow) {
                GKV_GDN_LAUNCH(kF16NarrowC)
            } else {
                GKV_GDN_LAUNCH(kFastC)
            }
#undef GKV_GDN_LAUNCH
        } else {
            switch (taps) {
                case 1: gdn_rollback_f32_kernel<1><<<blocks, kRollThreads, 0, st>>>(p); break;
                case 2: gdn_rollback_f32_kernel<2><<<blocks, kRollThreads, 0, st>>>(p); break;
                case 3: gdn_rollback_f32_kernel<3><<<blocks, kRollThreads, 0, st>>>(p); break;
                default: gdn_rollback_f32_kernel<4><<<blocks, kRollThreads, 0, st>>>(p); break;
            }
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return report_error(GKV_ERR_CUDA, "gdn_rollback launch: %s", cudaGetErrorString(e));
    }
    return GKV_OK;
}

}  // namespace
}  // namespace gkv

extern "C" int gkv_mtp_rollback(int32_t n_items, const int32_t *m, int32_t H, int32_t DK, int32_t DV,
                                int32_t C, const float *s0, const float *delta, const float *k,
                                const float *gcum, float *out, void *stream) {
    return gkv::mtp_rollback_impl<float>(n_items, m, H, DK, DV, C, s0, delta, k, gcum, out, stream);
}

extern "C" int gkv_mtp_rollback_f16(int32_t n_items, const int32_t *m, int32_t H, int32_t DK, int32_t DV,
                                    int32_t C, const void *s0, const float *delta, const float *k,
                                    const float *gcum, void *out, void *stream) {
    return gkv::mtp_rollback_impl<__half>(n_items, m, H, DK, DV, C, static_cast<const __half *>(s0), delta, k,
                                          gcum, static_cast<__half *>(out), stream);
}

extern "C" int gkv_gdn_rollback_f16(int32_t n_items, const int32_t *m, int32_t H, int32_t DK, int32_t DV,
                                    int32_t C, const void *s0, const float *delta, const float *k,
                                    const float *gcum, void *state_out, int32_t conv_dim, int32_t taps,
                                    const float *proj, const void *pre, void *conv_out, void *stream) {
    return gkv::gdn_rollback_impl<__half>(n_items, m, H, DK, DV, C, static_cast<const __half *>(s0), delta, k,
                                          gcum, static_cast<__half *>(state_out), conv_dim, taps, proj,
                                          static_cast<const __half *>(pre), static_cast<__half *>(conv_out), stream);
}

extern "C" int gkv_gdn_rollback(int32_t n_items, const int32_t *m, int32_t H, int32_t DK, int32_t DV, int32_t C,
                                const float *s0, const float *delta, const float *k, const float *gcum,
                                float *state_out, int32_t conv_dim, int32_t taps, const float *proj,
                                const float *pre, float *conv_out, void *stream) {
    return gkv::gdn_rollback_impl<float>(n_items, m, H, DK, DV, C, s0, delta, k, gcum, state_out, conv_dim, taps,
                                         proj, pre, conv_out, stream);
}

extern "C" int gkv_conv_rollback(int32_t n_items, const int32_t *m, int32_t conv_dim, int32_t taps, int32_t C,
                                 const float *proj, const float *pre, float *out, void *stream) {
    return gkv::conv_rollback_impl<float>(n_items, m, conv_dim, taps, C, proj, pre, out, stream);
}

extern "C" int gkv_conv_rollback_f16(int32_t n_items, const int32_t *m, int32_t conv_dim, int32_t taps,
                                     int32_t C, const float *proj, const void *pre, void *out, void *stream) {
    return gkv::conv_rollback_impl<__half>(n_items, m, conv_dim, taps, C, proj, static_cast<const __half *>(pre),
                                           static_cast<__half *>(out), stream);
}
