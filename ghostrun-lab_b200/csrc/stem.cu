// The policy's input stem on Blackwell tensor cores: NES colour numbers (+ per-line emphasis) of 4 frames -> palette
// RGB (bf16) -> 2x2 stride-2 convolution, 12 -> 16 channels, fused in one kernel (the reference runs it as a Triton
// kernel, rl/fused.py:36-96 _stem_inputs / _stem_fwd_kernel, called by rl/model.py:151-158 through fused_stem,
// rl/fused.py:163-169). The convolution reads every input pixel once, so it is a GEMM over output pixels:
//   out[p, o] = bias[o] + sum_k x[p, k] * W[o, k],  k = (frame * 3 + RGB) * 4 + dy * 2 + dx  (48 inputs)
// with x[p, k] the bf16 palette value of that input pixel's colour (palette index colour | emphasis << 6). Products
// are bf16 x bf16 summed in fp32 (tcgen05.mma kind::f16, fp32 accumulator in tensor memory); only the order of the
// fp32 additions can differ from another implementation of the same GEMM.
//
// Mapping: a CTA of 128 threads takes 128 output pixels (one M=128 tile) at a time. Each thread builds its pixel's
// 48 inputs (8 colour-number pairs + their emphasis, 24 palette lookups in shared memory) straight into the A tile in
// shared memory, laid out as 8x16-byte core matrices without swizzle (K-major: element (m, k) at
// (m / 8) * 768 + (m % 8) * 16 + (k / 8) * 128 + (k % 8) * 2); the weights (B, 16 x 48, same layout) stay in shared
// memory. One thread issues the three K=16 MMAs into 16 fp32 columns of tensor memory and commits them to an
// mbarrier; then warp w reads accumulator rows 32w..32w+31 (tcgen05.ld 32x32b), adds the bias and stores 16 bf16 per
// pixel (channels-last, 32 contiguous bytes). A tiles and accumulators are double-buffered, so one tile's MMAs run
// while the next is built. The kernel is HBM-bound (12-16 input bytes and 32 output bytes per output pixel against
// 1,536 flops); several persistent CTAs per SM keep loads in flight.
//
// The input is either the byte pictures [B, 4, 224, 240] or their 6-bit packed form [B, 4, 224, 180] (the rollout
// storage format, rl/csrc/rlenv.cu:126-134): the packed variant unpacks in the kernel.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstdint>
#include <string>

namespace {

constexpr int kH = 224, kW = 240, kOH = 112, kOW = 120, kFrames = 4;
constexpr int kTileM = 128, kK = 48, kN = 16;
constexpr int kThreads = 128;
constexpr unsigned kSpinLimit = 1u << 24;   // mbarrier polls before a tile is given up (error flag set)

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// Shared-memory matrix descriptor (no swizzle, K-major core matrices; Blackwell descriptor version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(lbo >> 4) << 16;
    d |= static_cast<uint64_t>(sbo >> 4) << 32;
    d |= 1ull << 46;   // version
    return d;          // base offset 0, relative leading offset, layout type 0 (no swizzle)
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both K-major, N = 16, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kN >> 3) << 17) |
                            (static_cast<uint32_t>(kTileM >> 4) << 24);

__device__ __forceinline__ uint32_t bf16_bits(float v) {
    return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
}

struct StemArgs {
    const uint8_t* obs;         // [B, 4, 224, 240] colour numbers, or [B, 4, 224, 180] packed 6-bit
    const uint8_t* emph;        // [B, 4, 224]
    const uint16_t* pal;        // [512][4] bf16 bits: R, G, B, 0 of colour | emphasis << 6
    const uint16_t* w;          // [16][48] bf16 bits, k = (frame * 3 + RGB) * 4 + dy * 2 + dx
    const uint16_t* bias;       // [16] bf16 bits
    uint16_t* out;              // [B, 112, 120, 16] bf16 bits
    int* err;                   // set to 1 when an MMA did not complete in time
    long long n_out;            // B * 112 * 120
};

// The raw inputs of one output pixel: for each (frame, dy) the two colour numbers (c0 | c1 << 8) and the emphasis.
struct Raw { uint32_t c[8]; uint32_t e[8]; };

template <bool PACKED>
__device__ __forceinline__ void load_raw(const StemArgs& a, long long p, Raw& r) {
    if (p >= a.n_out) {
#pragma unroll
        for (int q = 0; q < 8; ++q) { r.c[q] = 0; r.e[q] = 0; }
        return;
    }
    const uint32_t p32 = static_cast<uint32_t>(p);   // n_out < 2^31 (checked at launch): 32-bit constant divisions
    const uint32_t b = p32 / static_cast<uint32_t>(kOH * kOW);
    const uint32_t rr = p32 - b * static_cast<uint32_t>(kOH * kOW);
    const int oy = static_cast<int>(rr / kOW), ox = static_cast<int>(rr - (rr / kOW) * kOW);
#pragma unroll
    for (int f = 0; f < kFrames; ++f) {
#pragma unroll
        for (int dy = 0; dy < 2; ++dy) {
            const int q = f * 2 + dy;
            const long long plane_row = (static_cast<long long>(b) * kFrames + f) * kH + 2 * oy + dy;
            if constexpr (PACKED) {
                // the 3 bytes of 4-pixel group ox / 2 (rows are 4-byte aligned: 180 bytes); a second word only when the
                // group straddles two (then both lie inside the row)
                const long long off = plane_row * (kW / 4 * 3) + 3 * (ox >> 1);
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(a.obs + (off & ~3ll));
                const uint32_t lo = __ldg(wp), sh = static_cast<uint32_t>(off & 3) * 8u;
                const uint32_t hi = sh >= 16u ? __ldg(wp + 1) : 0u;
                const uint32_t v = __funnelshift_r(lo, hi, sh);
                const uint32_t s2 = (ox & 1) ? 12u : 0u;
                r.c[q] = ((v >> s2) & 63u) | (((v >> (s2 + 6)) & 63u) << 8);
            } else {
                const uint32_t two = __ldg(reinterpret_cast<const uint16_t*>(a.obs + plane_row * kW + 2 * ox));
                r.c[q] = two & 0x3F3Fu;
            }
            r.e[q] = static_cast<uint32_t>(__ldg(a.emph + plane_row)) << 6;
        }
    }
}

template <bool PACKED>
__global__ void __launch_bounds__(kThreads) k_stem_fwd(const __grid_constant__ StemArgs a) {
    __shared__ __align__(1024) uint8_t sA[2][kTileM * kK * 2];   // 2 x 12 KB (double-buffered A tiles)
    __shared__ __align__(128) uint8_t sB[kN * kK * 2];           // 1.5 KB
    __shared__ __align__(16) uint2 sPal[512];                    // 4 KB
    __shared__ float sBias[kN];
    __shared__ __align__(8) uint64_t mbar[2];
    __shared__ uint32_t tmem_base;
    __shared__ int bail;
    const int tid = threadIdx.x, warp = tid >> 5;

    for (int i = tid; i < 512; i += kThreads) sPal[i] = reinterpret_cast<const uint2*>(a.pal)[i];
    for (int i = tid; i < kN * kK; i += kThreads) {   // weights into the core-matrix layout (row n = output channel)
        const int n = i / kK, k = i % kK;
        const uint32_t off = (n / 8) * 768 + (n % 8) * 16 + (k / 8) * 128 + (k % 8) * 2;
        *reinterpret_cast<uint16_t*>(sB + off) = a.w[i];
    }
    if (tid < kN) sBias[tid] = __bfloat162float(__ushort_as_bfloat16(a.bias[tid]));
    if (tid == 0) {
        bail = 0;
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_u32(&mbar[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_u32(&mbar[1])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {   // 32 columns of tensor memory: two 16-column fp32 accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 32;" :: "r"(smem_u32(&tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    const uint32_t b_base = smem_u32(sB);
    uint32_t phase[2] = {0u, 0u};

    // Pipeline: iteration i builds tile i's A rows and issues its MMAs (buffer i % 2), then drains tile i - 1's
    // accumulator, so a tile's MMAs run while the next tile is built. Buffer reuse two iterations later is safe: its
    // MMAs were waited for (before the A rows are rewritten) and its accumulator reads finished (before the MMAs
    // that overwrite it, ordered by the barrier at the top of the iteration).
    const long long tiles = (a.n_out + kTileM - 1) / kTileM;
    long long prev_p = -1;
    int it = 0;
    for (long long tile = blockIdx.x;; tile += gridDim.x, ++it) {
        const bool have = tile < tiles;
        const int buf = it & 1;
        const long long p = tile * kTileM + tid;
        if (have) {
            Raw raw;
            load_raw<PACKED>(a, p, raw);
            uint32_t x[24];   // 48 bf16, two per word, k order
#pragma unroll
            for (int f = 0; f < kFrames; ++f) {
#pragma unroll
                for (int dy = 0; dy < 2; ++dy) {
                    const int q = f * 2 + dy;
                    const uint2 q0 = sPal[(raw.c[q] & 63u) | raw.e[q]], q1 = sPal[(raw.c[q] >> 8) | raw.e[q]];   // (R | G << 16, B)
                    // k = (f * 3 + ch) * 4 + dy * 2 + dx: the pair (dx = 0, 1) of channel ch is one 32-bit word
                    const int w0 = ((f * 3 + 0) * 4 + dy * 2) >> 1;
                    x[w0] = (q0.x & 0xFFFFu) | ((q1.x & 0xFFFFu) << 16);
                    x[w0 + 2] = (q0.x >> 16) | (q1.x & 0xFFFF0000u);
                    x[w0 + 4] = (q0.y & 0xFFFFu) | ((q1.y & 0xFFFFu) << 16);
                }
            }
            uint8_t* rowbase = sA[buf] + (tid / 8) * 768 + (tid % 8) * 16;   // 6 core-matrix rows of 16 bytes
#pragma unroll
            for (int j = 0; j < 6; ++j)
                *reinterpret_cast<uint4*>(rowbase + j * 128) = make_uint4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic-proxy stores -> tensor core reads
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        if (have && tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_base = smem_u32(sA[buf]);
            const uint32_t acc_cols = tmem + static_cast<uint32_t>(buf * kN);
#pragma unroll
            for (int kk = 0; kk < 3; ++kk) {   // K = 48 in three K = 16 steps (two 8-element core matrices each)
                const uint64_t da = smem_desc(a_base + kk * 256, 128, 768);
                const uint64_t db = smem_desc(b_base + kk * 256, 128, 768);
                const uint32_t acc = kk > 0 ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                    :: "r"(acc_cols), "l"(da), "l"(db), "r"(kIdesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         :: "r"(smem_u32(&mbar[buf])) : "memory");
        }
        if (it > 0) {   // ---- the previous tile: wait for its MMAs (bounded), bias, bf16, store
            const int pb = buf ^ 1;
            uint32_t done = 0;
            for (unsigned spin = 0; spin < kSpinLimit && !done; ++spin) {
                asm volatile("{\n\t.reg .pred q;\n\t"
                             "mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n\t"
                             "selp.u32 %0, 1, 0, q;\n\t}"
                             : "=r"(done) : "r"(smem_u32(&mbar[pb])), "r"(phase[pb]) : "memory");
            }
            phase[pb] ^= 1u;
            if (!done) bail = 1;
            __syncthreads();
            if (bail) {   // the tensor core did not answer: report and stop (tensor memory is freed below)
                if (tid == 0) atomicExch(a.err, 1);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint32_t d[16];
            const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(pb * kN);
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                         "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                         : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
                           "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15])
                         : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (prev_p >= 0 && prev_p < a.n_out) {
                uint32_t o[8];
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    const float lo = __uint_as_float(d[2 * n]) + sBias[2 * n];
                    const float hi = __uint_as_float(d[2 * n + 1]) + sBias[2 * n + 1];
                    o[n] = bf16_bits(lo) | (bf16_bits(hi) << 16);
                }
                uint4* dst = reinterpret_cast<uint4*>(a.out + prev_p * kN);
                dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
            }
        }
        if (!have) break;
        prev_p = p;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" :: "r"(tmem));
    }
}

thread_local std::string g_stem_error;

}  // namespace

extern "C" {

// Fused colour lookup + stem convolution (rl/fused.py:163-169 fused_stem semantics, forward). obs: [B,4,224,240]
// colour numbers (packed = 0) or [B,4,224,180] 6-bit packed pictures (packed = 1); emph [B,4,224]; pal4: [512][4]
// bf16 (R, G, B, 0 per palette index colour | emphasis << 6, the bf16-rounded palette); weight [16][48] bf16 (the
// conv weight [16,12,2,2] flattened); bias [16] bf16; out [B,112,120,16] bf16 (channels-last). err: device int, set
// to 1 if a tile's MMA did not complete (the call then still returns 0; read it after synchronising). Asynchronous
// on `stream`.
int rl_stem_fwd(const void* obs, const void* emph, const void* pal4, const void* weight, const void* bias, void* out,
                long long batch, int packed, int* err, void* stream) {
    StemArgs a;
    a.obs = static_cast<const uint8_t*>(obs);
    a.emph = static_cast<const uint8_t*>(emph);
    a.pal = static_cast<const uint16_t*>(pal4);
    a.w = static_cast<const uint16_t*>(weight);
    a.bias = static_cast<const uint16_t*>(bias);
    a.out = static_cast<uint16_t*>(out);
    a.err = err;
    a.n_out = batch * kOH * kOW;
    if (batch <= 0) return 0;
    if (a.n_out >= (1ll << 31)) { g_stem_error = "rl_stem_fwd: batch too large (B * 112 * 120 must be below 2^31)"; return 1; }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long tiles = (a.n_out + kTileM - 1) / kTileM;
    const long long want = static_cast<long long>(sms) * 6;   // persistent CTAs, 6 per SM (30 KB shared each)
    const unsigned grid = static_cast<unsigned>(tiles < want ? tiles : want);
    auto s = static_cast<cudaStream_t>(stream);
    if (packed) k_stem_fwd<true><<<grid, kThreads, 0, s>>>(a);
    else k_stem_fwd<false><<<grid, kThreads, 0, s>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { g_stem_error = cudaGetErrorString(e); return 1; }
    return 0;
}

const char* rl_stem_error(void) { return g_stem_error.c_str(); }

}  // extern "C"
