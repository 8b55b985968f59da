// The policy's input stem on Blackwell tensor cores: NES colour numbers (+ per-line emphasis) of 4 frames -> palette
// RGB (bf16) -> 2x2 stride-2 convolution, 12 -> 16 channels, fused in one kernel (the reference runs it as a Triton
// kernel, rl/fused.py:36-96 _stem_inputs / _stem_fwd_kernel, called by rl/model.py:151-158 through fused_stem,
// rl/fused.py:163-169). The convolution reads every input pixel once, so it is a GEMM over output pixels:
//   out[p, o] = bias[o] + sum_k x[p, k] * W[o, k],  k = (frame * 3 + RGB) * 4 + dy * 2 + dx  (48 inputs)
// with x[p, k] the bf16 palette value of that input pixel's colour (palette index colour | emphasis << 6). Products
// are bf16 x bf16 summed in fp32 (tcgen05.mma kind::f16, fp32 accumulator in tensor memory); only the order of the
// fp32 additions can differ from another implementation of the same GEMM.
//
// Mapping: a CTA of 128 threads takes one output row (120 pixels; an M=128 tile whose rows 120..127 idle) at a time.
// The row's input is exactly 8 picture rows (4 frames x 2 rows); the whole CTA loads them with coalesced 4-byte loads
// one tile ahead (held in registers, then staged in shared memory). The K order of the GEMM is permuted so that a
// palette lookup lands in the A operand unchanged: k' = pos * 4 + c, pos = frame * 4 + dy * 2 + dx (16 input pixels),
// c = R, G, B, 1 (64 inputs); the weights are permuted the same way, the constant-1 input of position 0 carries the
// bias and the others weigh 0. Thread m looks up its pixel's 16 palette entries (8 bytes each, shared memory) and
// writes them as its row of A in tensor memory (tcgen05.st 32x32b: warp w owns lanes 32w..32w+31). One thread issues
// the four K=16 MMAs (A from tensor memory, weights from shared memory as no-swizzle K-major core matrices: element
// (n, k') at (n / 8) * 1024 + (n % 8) * 16 + (k' / 8) * 128 + (k' % 8) * 2) into 16 fp32 columns and commits them to
// an mbarrier. The next iteration waits for them (bounded), reads the accumulator (tcgen05.ld 32x32b), writes the
// next tile's A, and the row's 120 x 16 bf16 outputs (channels-last, 3,840 contiguous bytes) are stored while the
// tensor core works. The kernel moves 12-16 input bytes and 32 output bytes per output pixel against 2,048 flops.
//
// The input is either the byte pictures [B, 4, 224, 240] or their 6-bit packed form [B, 4, 224, 180] (the rollout
// storage format, rl/csrc/rlenv.cu:126-134): the packed variant unpacks in the kernel.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstdint>
#include <string>
#include "../../include/rlenv_api.h"   // rl_stem_* compiled against their C-ABI declarations

namespace {

constexpr int kH = 224, kW = 240, kOH = 112, kOW = 120, kFrames = 4;
constexpr int kTileM = 128, kK = 48, kKp = 64, kN = 16;   // kKp: the permuted K (16 input pixels x R, G, B, 1)
constexpr uint32_t kAccCol = 32;                          // accumulator columns 32..47; A rows in columns 0..31
constexpr uint32_t kOneBf16 = 0x3F80u;                    // 1.0 in bf16
constexpr int kThreads = 128;
constexpr int kCtasPerSm = 8;
constexpr size_t kPadSmem = 16 * 1024;   // with ~10.3 KB static: 26.5 KB per CTA, at most 8 CTAs per SM
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

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
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

// The 8 picture rows of one output row, loaded by the whole CTA one tile ahead: 4-byte words in registers, then
// shared memory (rows at a 256-byte stride), and the rows' emphasis bits (as palette offsets, emphasis << 6).
template <bool PACKED>
struct RowLoad {
    static constexpr int kRowBytes = PACKED ? kW / 4 * 3 : kW;   // 180 or 240
    static constexpr int kWords = kRowBytes / 4;                  // 45 or 60 per picture row
    static constexpr int kPer = (8 * kWords + kThreads - 1) / kThreads;   // words per thread (3 or 4)
    uint32_t w[kPer];
    uint32_t e;   // thread q < 8: picture row q = frame * 2 + dy
};

template <bool PACKED>
__device__ __forceinline__ void rows_load(const StemArgs& a, long long r, long long rows, int tid, RowLoad<PACKED>& L) {
    using R = RowLoad<PACKED>;
    if (r >= rows) return;
    const uint32_t r32 = static_cast<uint32_t>(r);   // rows < 2^31 / 120 (checked at launch)
    const uint32_t b = r32 / kOH, oy = r32 - b * kOH;
#pragma unroll
    for (int k = 0; k < R::kPer; ++k) {
        const int wi = tid + k * kThreads;
        if (wi < 8 * R::kWords) {
            const int q = wi / R::kWords, c = wi - q * R::kWords;
            const long long row = (static_cast<long long>(b) * kFrames + (q >> 1)) * kH + 2 * oy + (q & 1);
            L.w[k] = __ldg(reinterpret_cast<const uint32_t*>(a.obs + row * R::kRowBytes) + c);
        }
    }
    if (tid < 8) {
        const long long row = (static_cast<long long>(b) * kFrames + (tid >> 1)) * kH + 2 * oy + (tid & 1);
        L.e = static_cast<uint32_t>(__ldg(a.emph + row)) << 6;
    }
}

template <bool PACKED>
__device__ __forceinline__ void rows_store(const RowLoad<PACKED>& L, uint32_t* rowbuf, uint32_t* ebuf, int tid) {
    using R = RowLoad<PACKED>;
#pragma unroll
    for (int k = 0; k < R::kPer; ++k) {
        const int wi = tid + k * kThreads;
        if (wi < 8 * R::kWords) {
            const int q = wi / R::kWords, c = wi - q * R::kWords;
            rowbuf[q * 64 + c] = L.w[k];
        }
    }
    if (tid < 8) ebuf[tid] = L.e;
}

// Half of a pixel's A row (picture rows q0..q0+3: 8 input pixels, 16 words) from the staged rows: two palette
// lookups per picture row, each (R | G << 16, B | 1.0 << 16) from two 4-byte tables. A picture row has one emphasis
// for the whole block, so its lookups fall in one 64-entry slice: as 4-byte words that slice puts at most 2 colours
// on a shared-memory bank (as 8-byte entries, 4 colours shared a bank pair).
template <bool PACKED>
__device__ __forceinline__ void build_half(const uint32_t* rb, const uint32_t* eb, const uint32_t* pal_rg,
                                           const uint32_t* pal_b1, int q0, uint32_t wi, uint32_t sh, uint32_t* x) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int q = q0 + j;
        uint32_t c0, c1;
        if constexpr (PACKED) {   // the pair's 12 bits at bit 12 * ox of the row (a little-endian 6-bit stream)
            const uint32_t v = __funnelshift_r(rb[q * 64 + wi], rb[q * 64 + wi + 1], sh);
            c0 = v & 63u;
            c1 = (v >> 6) & 63u;
        } else {                  // bytes 2 * ox, 2 * ox + 1
            const uint32_t v = rb[q * 64 + wi] >> sh;
            c0 = v & 63u;
            c1 = (v >> 8) & 63u;
        }
        const uint32_t e = eb[q];
        const uint32_t i0 = c0 | e, i1 = c1 | e;
        x[4 * j] = pal_rg[i0];
        x[4 * j + 1] = pal_b1[i0];
        x[4 * j + 2] = pal_rg[i1];
        x[4 * j + 3] = pal_b1[i1];
    }
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* x) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                 "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
                 :: "r"(taddr), "r"(x[0]), "r"(x[1]), "r"(x[2]), "r"(x[3]), "r"(x[4]), "r"(x[5]), "r"(x[6]), "r"(x[7]),
                    "r"(x[8]), "r"(x[9]), "r"(x[10]), "r"(x[11]), "r"(x[12]), "r"(x[13]), "r"(x[14]), "r"(x[15])
                 : "memory");
}

// Bounded wait for phase `parity` of the mbarrier: 1 when it completed.
__device__ __forceinline__ uint32_t mbar_wait(uint32_t addr, uint32_t parity) {
    uint32_t done = 0;
    for (unsigned spin = 0; spin < kSpinLimit && !done; ++spin) {
        asm volatile("{\n\t.reg .pred q;\n\t"
                     "mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, q;\n\t}"
                     : "=r"(done) : "r"(addr), "r"(parity) : "memory");
    }
    return done;
}

template <bool PACKED>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) k_stem_fwd(const __grid_constant__ StemArgs a) {
    __shared__ __align__(128) uint8_t sB[kN * kKp * 2];   // 2 KB: permuted weights + bias
    __shared__ __align__(16) uint32_t sPalRG[512];       // 2 KB: R | G << 16
    __shared__ __align__(16) uint32_t sPalB1[512];       // 2 KB: B | 1.0 << 16
    __shared__ __align__(16) uint32_t sRow[2][8 * 64];    // 2 x 2 KB: a tile's 8 picture rows
    __shared__ __align__(16) uint32_t sEmph[2][8];
    __shared__ __align__(8) uint64_t mbar;
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5;

    for (int i = tid; i < 512; i += kThreads) {
        const uint2 v = reinterpret_cast<const uint2*>(a.pal)[i];
        sPalRG[i] = v.x;                                   // R | G << 16
        sPalB1[i] = (v.y & 0xFFFFu) | (kOneBf16 << 16);    // B | 1.0 << 16
    }
    for (int i = tid; i < kN * kKp; i += kThreads) {   // permuted weights into the core-matrix layout (row n = channel)
        const int n = i / kKp, kp = i % kKp, pos = kp >> 2, c = kp & 3;
        const int f = pos >> 2, dy = (pos >> 1) & 1, dx = pos & 1;
        const uint16_t v = c < 3 ? a.w[n * kK + (f * 3 + c) * 4 + dy * 2 + dx] : (pos == 0 ? a.bias[n] : uint16_t(0));
        *reinterpret_cast<uint16_t*>(sB + (n / 8) * 1024 + (n % 8) * 16 + (kp / 8) * 128 + (kp % 8) * 2) = v;
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_u32(&mbar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {   // 64 columns of tensor memory: A rows (32 columns of bf16 pairs) and the fp32 accumulator (16)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 64;" :: "r"(smem_u32(&tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    const long long rows = a.n_out / kOW;   // tiles: output rows
    const long long step = gridDim.x;
    RowLoad<PACKED> L;
    rows_load<PACKED>(a, blockIdx.x, rows, tid, L);          // tile 0's rows
    rows_store<PACKED>(L, sRow[0], sEmph[0], tid);
    rows_load<PACKED>(a, blockIdx.x + step, rows, tid, L);   // tile 1's rows, in flight
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    const uint32_t lane_a = tmem + (static_cast<uint32_t>(warp * 32) << 16);   // this warp's lanes, column 0
    const uint32_t b_base = smem_u32(&sB[0]);
    const uint32_t bar = smem_u32(&mbar);
    // where this thread's pixel pair sits in a staged picture row
    const int ox = tid < kOW ? tid : kOW - 1;
    const uint32_t bit = PACKED ? 12u * static_cast<uint32_t>(ox) : 16u * static_cast<uint32_t>(ox);
    const uint32_t wi = bit >> 5, sh = bit & 31u;
    uint32_t phase = 0;

    // Iteration i (tile r, row buffer i % 2): wait for tile i-1's MMAs; look up tile i's inputs and write them as
    // A rows; read tile i-1's accumulator; stage tile i+1's rows; barrier; MMAs of tile i; store tile i-1's outputs;
    // issue the loads of tile i+2. Row buffer i % 2 is rewritten (iteration i+1) only after the barrier that follows
    // its reads; A and the accumulator are rewritten only after the MMAs that read or wrote them completed.
    long long prev_r = -1;
    int it = 0;
    for (long long r = blockIdx.x;; r += step, ++it) {
        const bool have = r < rows;
        const int buf = it & 1;
        uint32_t ok = 1, d[16];
        if (it > 0) ok = mbar_wait(bar, phase);   // tile i-1's MMAs (they read A and wrote the accumulator)
        if (have && ok) {
            uint32_t x[16];
            build_half<PACKED>(sRow[buf], sEmph[buf], sPalRG, sPalB1, 0, wi, sh, x);
            tmem_st16(lane_a, x);
            build_half<PACKED>(sRow[buf], sEmph[buf], sPalRG, sPalB1, 4, wi, sh, x);
            tmem_st16(lane_a + 16, x);
        }
        if (it > 0) {
            phase ^= 1u;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                         "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                         : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
                           "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15])
                         : "r"(lane_a + kAccCol));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        }
        if (have && ok) {
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            if (r + step < rows) rows_store<PACKED>(L, sRow[buf ^ 1], sEmph[buf ^ 1], tid);   // tile i+1's rows
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        const int fail = __syncthreads_or(ok == 0u);
        if (fail) {   // the tensor core did not answer: report, wait (bounded) for the MMAs in flight, stop
            if (tid == 0) atomicExch(a.err, 1);
            mbar_wait(bar, phase ^ 1u);
            break;    // tensor memory is freed below
        }
        if (have && tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int kk = 0; kk < kKp / 16; ++kk) {   // K' = 64 in four K = 16 steps (8 columns of A each)
                const uint64_t db = smem_desc(b_base + kk * 256, 128, 1024);
                const uint32_t acc = kk > 0 ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                    :: "r"(tmem + kAccCol), "r"(tmem + static_cast<uint32_t>(kk * 8)), "l"(db), "r"(kIdesc), "r"(acc),
                       "r"(0u), "r"(0u), "r"(0u), "r"(0u));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         :: "r"(bar) : "memory");
        }
        if (it > 0 && tid < kOW) {   // tile i-1: bf16 outputs (the bias is in the sum)
            uint32_t o[8];
#pragma unroll
            for (int n = 0; n < 8; ++n) o[n] = bf16x2_bits(__uint_as_float(d[2 * n]), __uint_as_float(d[2 * n + 1]));
            uint4* dst = reinterpret_cast<uint4*>(a.out + (prev_r * kOW + tid) * kN);
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
        if (!have) break;
        rows_load<PACKED>(a, r + 2 * step, rows, tid, L);   // tile i+2's rows in flight
        prev_r = r;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 64;" :: "r"(tmem));
    }
}

// ------------------------------------------------------------------------------------------------ backward
// dW = sum_p g[p] x[p]^T and dbias = sum_p g[p] over the output pixels p (the reference's _stem_bwd_kernel,
// rl/fused.py:89-107; the input pictures are not trained). On the tensor cores with K = pixels: A = x^T (M = the 64
// permuted inputs k', padded to M = 128 with zero rows), B = g (N = 16 channels), D = dW^T in tensor memory,
// accumulated over all of a CTA's tiles. Both operands are MN-major no-swizzle core matrices: pixel p's 64 inputs
// are 8 chunks of 16 bytes, chunk c of A at c * 2048 + (p / 8) * 128 + (p % 8) * 16; g's 16 channels are 2 chunks
// of B at the same places. A's padding rows 64..127 (chunks 8..15) are whatever shared memory follows the buffer:
// they only reach D rows 64..127, which are never read. The constant-1 input of position 0 (k' = 3) makes
// D row 3 the bias gradient. Tiles are output rows (120 pixels, 8 zero rows of g); each CTA writes its 64 x 16
// partial sums, and k_stem_bwd_reduce adds the CTAs' partials in a fixed order into dW [16][48] and dbias [16].
constexpr uint32_t kBwdChunk = 2048;                    // bytes between core-matrix columns along M / N
constexpr int kBwdCtasPerSm = 4;
constexpr uint32_t kBwdA = 8 * kBwdChunk;               // 16 KB per A buffer (its 8 chunks of inputs)
constexpr uint32_t kBwdB = 2 * kBwdChunk;               // 4 KB per B buffer
constexpr uint32_t kBwdSmem = 2 * kBwdA + 2 * kBwdB + 4096 + 2 * 2048 + 64 + 64;
// the M = 128 operand of buffer 1 reaches 16 KB past its 8 chunks: into the buffers and tables after it
static_assert(kBwdSmem >= 3 * kBwdA, "A's padding rows must stay inside the block's shared memory");
// kind::f16, fp32 D, bf16 A and B, both MN-major (bits 15, 16), N = 16, M = 128
constexpr uint32_t kIdescBwd = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
                               (static_cast<uint32_t>(kN >> 3) << 17) | (static_cast<uint32_t>(kTileM >> 4) << 24);

struct StemBwdArgs {
    const uint8_t* obs;
    const uint8_t* emph;
    const uint16_t* pal;
    const uint16_t* g;          // [B, 112, 120, 16] bf16 bits: the output gradient
    float* part;                // [grid][64][16] per-CTA dW^T partial sums
    int* err;
    long long n_out;
};

template <bool PACKED>
__global__ void __launch_bounds__(kThreads) k_stem_bwd(const __grid_constant__ StemBwdArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* sA = smem;                                                    // [2][kBwdA]
    uint8_t* sB = smem + 2 * kBwdA;                                        // [2][kBwdB]
    uint32_t* sPalRG = reinterpret_cast<uint32_t*>(sB + 2 * kBwdB);        // [512] R | G << 16
    uint32_t* sPalB1 = sPalRG + 512;                                       // [512] B | 1.0 << 16
    uint32_t* sRow = reinterpret_cast<uint32_t*>(sB + 2 * kBwdB + 4096);   // [2][8 * 64]
    uint32_t* sEmph = sRow + 2 * 8 * 64;                                   // [2][8]
    __shared__ __align__(8) uint64_t mbar[2];
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5;

    for (int i = tid; i < 512; i += kThreads) {
        const uint2 v = reinterpret_cast<const uint2*>(a.pal)[i];
        sPalRG[i] = v.x;
        sPalB1[i] = (v.y & 0xFFFFu) | (kOneBf16 << 16);
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_u32(&mbar[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_u32(&mbar[1])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 32;" :: "r"(smem_u32(&tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    const long long rows = a.n_out / kOW;
    const long long step = gridDim.x;
    StemArgs fa;   // the input side shares the forward's row loads
    fa.obs = a.obs; fa.emph = a.emph;
    RowLoad<PACKED> L;
    rows_load<PACKED>(fa, blockIdx.x, rows, tid, L);
    rows_store<PACKED>(L, sRow, sEmph, tid);
    rows_load<PACKED>(fa, blockIdx.x + step, rows, tid, L);
    // the output gradient of the next tile, one tile ahead (pixels 120..127 weigh nothing)
    auto g_load = [&](long long r, uint4& q0, uint4& q1) {
        q0 = make_uint4(0u, 0u, 0u, 0u);
        q1 = q0;
        if (tid < kOW && r < rows) {
            const uint4* gp = reinterpret_cast<const uint4*>(a.g + (r * kOW + tid) * kN);
            q0 = __ldg(gp);
            q1 = __ldg(gp + 1);
        }
    };
    uint4 g0, g1;
    g_load(blockIdx.x, g0, g1);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;
    const int ox = tid < kOW ? tid : kOW - 1;
    const uint32_t bit = PACKED ? 12u * static_cast<uint32_t>(ox) : 16u * static_cast<uint32_t>(ox);
    const uint32_t wi = bit >> 5, sh = bit & 31u;
    const uint32_t cm = (static_cast<uint32_t>(tid) / 8) * 128 + (static_cast<uint32_t>(tid) % 8) * 16;   // this pixel's row
    uint32_t phase[2] = {0u, 0u};
    int fail = 0;
    int it = 0;
    for (long long r = blockIdx.x; r < rows; r += step, ++it) {
        const int buf = it & 1;
        uint32_t ok = 1;
        if (it >= 2) {   // tile it-2 read this buffer
            ok = mbar_wait(smem_u32(&mbar[buf]), phase[buf]);
            if (ok) phase[buf] ^= 1u;
        }
        if (ok) {
            uint8_t* A = sA + buf * kBwdA;
            uint32_t x[16];
            build_half<PACKED>(sRow + buf * 8 * 64, sEmph + buf * 8, sPalRG, sPalB1, 0, wi, sh, x);
#pragma unroll
            for (int c = 0; c < 4; ++c)
                *reinterpret_cast<uint4*>(A + c * kBwdChunk + cm) = make_uint4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
            build_half<PACKED>(sRow + buf * 8 * 64, sEmph + buf * 8, sPalRG, sPalB1, 4, wi, sh, x);
#pragma unroll
            for (int c = 0; c < 4; ++c)
                *reinterpret_cast<uint4*>(A + (4 + c) * kBwdChunk + cm) = make_uint4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
            uint8_t* Bb = sB + buf * kBwdB;
            *reinterpret_cast<uint4*>(Bb + cm) = g0;
            *reinterpret_cast<uint4*>(Bb + kBwdChunk + cm) = g1;
            if (r + step < rows) rows_store<PACKED>(L, sRow + (buf ^ 1) * 8 * 64, sEmph + (buf ^ 1) * 8, tid);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        fail = __syncthreads_or(ok == 0u);
        if (fail) break;
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_base = smem_u32(sA + buf * kBwdA), b_base = smem_u32(sB + buf * kBwdB);
#pragma unroll
            for (int ks = 0; ks < kTileM / 16; ++ks) {   // 8 steps of 16 pixels
                const uint64_t da = smem_desc(a_base + ks * 256, 128, kBwdChunk);
                const uint64_t db = smem_desc(b_base + ks * 256, 128, kBwdChunk);
                const uint32_t acc = (it > 0 || ks > 0) ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                    :: "r"(tmem), "l"(da), "l"(db), "r"(kIdescBwd), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         :: "r"(smem_u32(&mbar[buf])) : "memory");
        }
        rows_load<PACKED>(fa, r + 2 * step, rows, tid, L);
        g_load(r + step, g0, g1);
    }
    // drain (also after a failure): the MMAs of the last two tiles issued, bounded; then rows 0..63 of D (warps 0
    // and 1) to this CTA's partial
    uint32_t ok = 1;
    for (int k = 1; k <= 2; ++k) {
        const int j = it - k;
        if (j >= 0) ok &= mbar_wait(smem_u32(&mbar[j & 1]), phase[j & 1]);
    }
    if (__syncthreads_or(fail != 0 || ok == 0u)) {
        if (tid == 0) atomicExch(a.err, 1);
    } else if (it > 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (warp < 2) {
            uint32_t d[16];
            const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                         "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                         : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
                           "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15])
                         : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            float4* dst = reinterpret_cast<float4*>(a.part + (static_cast<size_t>(blockIdx.x) * 64 + tid) * kN);
#pragma unroll
            for (int q = 0; q < 4; ++q)
                dst[q] = make_float4(__uint_as_float(d[4 * q]), __uint_as_float(d[4 * q + 1]),
                                     __uint_as_float(d[4 * q + 2]), __uint_as_float(d[4 * q + 3]));
        }
    } else if (tid < 64) {   // no tile: a zero partial
        float4* dst = reinterpret_cast<float4*>(a.part + (static_cast<size_t>(blockIdx.x) * 64 + tid) * kN);
        for (int q = 0; q < 4; ++q) dst[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" :: "r"(tmem));
    }
}

// dW[o][k] and dbias[o] from the CTAs' partials (fixed order): k = (frame * 3 + c) * 4 + dy * 2 + dx is row
// k' = (frame * 4 + dy * 2 + dx) * 4 + c of D; dbias is row 3.
__global__ void k_stem_bwd_reduce(const float* part, int parts, float* dw, float* db) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // 16 * 48 weights, then 16 biases
    if (i >= kN * kK + kN) return;
    int row, o;
    if (i < kN * kK) {
        o = i / kK;
        const int k = i % kK, c = (k / 4) % 3, f = k / 12, pos = f * 4 + (k % 4);
        row = pos * 4 + c;
    } else {
        o = i - kN * kK;
        row = 3;
    }
    float s = 0.f;
    for (int p = 0; p < parts; ++p) s += part[(static_cast<size_t>(p) * 64 + row) * kN + o];
    if (i < kN * kK) dw[i] = s;
    else db[o] = s;
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
    if ((reinterpret_cast<uintptr_t>(obs) & 3) || (reinterpret_cast<uintptr_t>(out) & 15)) {
        g_stem_error = "rl_stem_fwd: obs must be 4-byte and out 16-byte aligned";
        return 1;
    }
    const long long tiles = batch * kOH;   // output rows
    // persistent CTAs, 8 per SM: 8 x 64 columns fill the SM's tensor memory; the unused dynamic shared memory keeps a
    // ninth CTA off the SM (its allocation would wait for a CTA to finish)
    const long long want = static_cast<long long>(sms) * kCtasPerSm;
    const unsigned grid = static_cast<unsigned>(tiles < want ? tiles : want);
    auto s = static_cast<cudaStream_t>(stream);
    if (packed) k_stem_fwd<true><<<grid, kThreads, kPadSmem, s>>>(a);
    else k_stem_fwd<false><<<grid, kThreads, kPadSmem, s>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { g_stem_error = cudaGetErrorString(e); return 1; }
    return 0;
}

const char* rl_stem_error(void) { return g_stem_error.c_str(); }

// Work space of rl_stem_bwd on the current device: the CTAs' partial sums (64 x 16 fp32 each, 4 CTAs per SM).
size_t rl_stem_bwd_work_bytes(void) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return static_cast<size_t>(sms) * kBwdCtasPerSm * 64 * kN * sizeof(float);
}

// Stem backward (rl/fused.py:130-160 stem_bwd semantics): grad [B,112,120,16] bf16 (channels-last), the forward's
// obs / emph / pal4 -> dw [16][48] fp32 (the conv weight's gradient, flattened as the forward's weight) and db [16]
// fp32. work: device memory of rl_stem_bwd_work_bytes() bytes. err as in rl_stem_fwd. Asynchronous on `stream`.
int rl_stem_bwd(const void* grad, const void* obs, const void* emph, const void* pal4, void* dw, void* db,
                long long batch, int packed, void* work, size_t work_bytes, int* err, void* stream) {
    StemBwdArgs a;
    a.obs = static_cast<const uint8_t*>(obs);
    a.emph = static_cast<const uint8_t*>(emph);
    a.pal = static_cast<const uint16_t*>(pal4);
    a.g = static_cast<const uint16_t*>(grad);
    a.part = static_cast<float*>(work);
    a.err = err;
    a.n_out = batch * kOH * kOW;
    if (batch <= 0) {
        g_stem_error = "rl_stem_bwd: batch must be positive";
        return 1;
    }
    if (a.n_out >= (1ll << 31)) { g_stem_error = "rl_stem_bwd: batch too large (B * 112 * 120 must be below 2^31)"; return 1; }
    if ((reinterpret_cast<uintptr_t>(obs) & 3) || (reinterpret_cast<uintptr_t>(grad) & 15) ||
        (reinterpret_cast<uintptr_t>(work) & 15)) {
        g_stem_error = "rl_stem_bwd: obs must be 4-byte, grad and work 16-byte aligned";
        return 1;
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long tiles = batch * kOH;
    const long long want = static_cast<long long>(sms) * kBwdCtasPerSm;
    const unsigned grid = static_cast<unsigned>(tiles < want ? tiles : want);
    if (work_bytes < static_cast<size_t>(grid) * 64 * kN * sizeof(float)) {
        g_stem_error = "rl_stem_bwd: work space smaller than rl_stem_bwd_work_bytes()";
        return 1;
    }
    auto s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (packed) {
        e = cudaFuncSetAttribute(k_stem_bwd<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kBwdSmem));
        if (e == cudaSuccess) k_stem_bwd<true><<<grid, kThreads, kBwdSmem, s>>>(a);
    } else {
        e = cudaFuncSetAttribute(k_stem_bwd<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kBwdSmem));
        if (e == cudaSuccess) k_stem_bwd<false><<<grid, kThreads, kBwdSmem, s>>>(a);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e == cudaSuccess) {
        k_stem_bwd_reduce<<<(kN * kK + kN + 255) / 256, 256, 0, s>>>(a.part, static_cast<int>(grid), static_cast<float*>(dw),
                                                                      static_cast<float*>(db));
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) { g_stem_error = cudaGetErrorString(e); return 1; }
    return 0;
}

}  // extern "C"
