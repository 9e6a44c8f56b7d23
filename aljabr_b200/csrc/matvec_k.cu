// Batch-1 GGUF K-quant dequantise-and-matvec (y = W x) for Q4_K and Q6_K,
// the 256-value super-block formats the reference's raw rows serve with
// GgufQ4RawDot.dotRowQ4K and GgufQ6RawDot.dotRowQ6K
// (engine/gguf/aljabr-gguf-core/.../runtime/GgufQ4RawDot.java:38-141,
// GgufQ6RawDot.java:33-133,403-513; block layouts in GgufQuantFormats.java:51-53
// and GgufKQuantLayout.java:37-66).
//
// Q4_K (144 B): fp16 d, fp16 dmin, 12 bytes of packed 6-bit (scale, min)
// pairs for 8 sub-blocks of 32, 128 bytes of nibbles; value 64j + t is the
// low (t < 32) or high nibble of byte 32j + t % 32, times d*scale, minus
// dmin*min of sub-block 2j + (t >= 32).
// Q6_K (210 B): ql[128], qh[64], int8 scales[16], fp16 d at byte 208; in
// half h, value 32k + i is nibble (k >> 1) of ql[64h + 32(k & 1) + i] with
// bits 2k..2k+1 of qh[32h + i] above it, minus 32, times
// d*scales[8h + 2k + i/16].
//
// A CTA serves 4 consecutive rows (8 for Q4_K with K <= 4096); its 8 warps deal out "tasks" (a few
// blocks of one row subset) and meet in shared memory at the end, summed in
// fixed order (deterministic).  Within a task consecutive lanes read
// consecutive code bytes, and each lane loads its x values once for all the
// rows it walks:
//   * Q4_K: a task is 4 blocks x RS rows; lane (block, c) takes code bytes
//     16c..16c+15, i.e. 16 values of each of sub-blocks 2(c/2) and 2(c/2) + 1,
//     so one header decode serves 32 values;
//   * Q6_K blocks are only 2-byte aligned (210 B): a task is one block x 2 RS
//     rows; lane (row half, h, i0) takes positions i0..i0+3 of half h, i.e.
//     two ql words and one qh word for 16 values.
// A code becomes a float by OR-ing it into the mantissa of 2^(23 - p), p its
// own bit position in the fetched word, and subtracting (exact, one LOP3 per
// value and one packed subtract per two; no shifts for most positions); the
// multiply-adds run on packed f32x2 pairs.  The row bytes are read once, and
// one thread per CTA prefetches the CTA's contiguous row range into L2.
#include "common.cuh"

namespace alj {
namespace {

constexpr int kKWarps = 8;
constexpr int kKRows = 4;     // rows per CTA

// L2 prefetch of the 16-byte-aligned inside of [base, base + bytes), in
// 16 KB bulk requests: the CTA's rows are one contiguous range, and one
// thread puts all of it in flight at once, so the warps' own loads find it
// in L2 instead of each paying the HBM round trip in turn.
__device__ __forceinline__ void prefetch_rows_l2(const uint8_t* base, size_t bytes) {
    uintptr_t a = (reinterpret_cast<uintptr_t>(base) + 15) & ~uintptr_t(15);
    const uintptr_t end = (reinterpret_cast<uintptr_t>(base) + bytes) & ~uintptr_t(15);
    for (; a + 16 <= end; a += 16384) {
        const uintptr_t left = end - a;
        const uint32_t n = static_cast<uint32_t>(left < 16384 ? left : 16384) & ~15u;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
    }
}

struct KRows {
    const uint8_t* w;
    const float* x;
    float* y;
    const float* bias;
    const float* residual;
    int K, N;
};

// Float bit patterns of 2^(23 - p): OR-ing a 4-bit code c into mantissa bits
// p..p+3 of one gives 2^(23 - p) + c exactly, for any p <= 19.
constexpr uint32_t kMag0 = 150u << 23, kMag4 = 146u << 23, kMag8 = 142u << 23, kMag12 = 138u << 23,
                   kMag16 = 134u << 23;

// (scale, min) of Q4_K sub-blocks 2j and 2j + 1 as 16-bit byte pairs, from the
// block header hd (bytes 4..15 hold the packed 6-bit pairs): sub-block i < 4
// keeps its scale in the low 6 bits of byte 4 + i and its min in byte 8 + i;
// i >= 4 has the low 4 bits in byte 8 + i and the top 2 in bytes i and 4 + i.
__device__ __forceinline__ void q4k_pair_scales(const uint4& hd, int j, uint32_t& sp, uint32_t& mp) {
    const int sh = 16 * (j & 1);
    const uint32_t Y = hd.y >> sh, Z = hd.z >> sh, W = hd.w >> sh;
    const uint32_t s_lo = Y & 0x3F3Fu, m_lo = Z & 0x3F3Fu;
    const uint32_t s_hi = (W & 0x0F0Fu) | ((Y >> 2) & 0x3030u);
    const uint32_t m_hi = ((W >> 4) & 0x0F0Fu) | ((Z >> 2) & 0x3030u);
    sp = j >= 2 ? s_hi : s_lo;
    mp = j >= 2 ? m_hi : m_lo;
}

// Q4_K: lane (bl, c) of a warp task takes code bytes 16c..16c+15 of block
// 4 g + bl: low nibbles are elements 16 (c & 1) + k of sub-block 2 (c >> 1),
// high nibbles the same elements of sub-block 2 (c >> 1) + 1.  The 32 x values
// (and their two sums) are loaded once per task and serve the task's RS rows.
// Each nibble becomes a float with one LOP3 into the mantissa of 2^(23 - p) at
// its own bit position p (no shifts for bytes 0..2) and one packed subtract.
template <int R, int RS>
__global__ void __launch_bounds__(kKWarps * 32, 3) q4k_matvec_kernel(const KRows p) {
    pdl_launch_dependents();
    constexpr int kSub = R / RS;   // row subsets; warp w always serves subset w % kSub
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * R;
    const int nb = p.K / 256;
    const size_t row_bytes = static_cast<size_t>(nb) * 144;
    // the weights never depend on the previous kernel: their L2 prefetch goes
    // out before the wait for x
    if (threadIdx.x == 0) prefetch_rows_l2(p.w + row0 * row_bytes, min(R, p.N - row0) * row_bytes);
    pdl_wait();   // x may come from the previous kernel
    const int bl = lane >> 3, c = lane & 7, j = c >> 1;
    const int sub = warp % kSub;
    const uint8_t* rowp[RS];
#pragma unroll
    for (int r = 0; r < RS; ++r)
        rowp[r] = p.w + static_cast<size_t>(min(row0 + sub * RS + r, p.N - 1)) * row_bytes + 16 + 16 * c;
    const f2 offA01 = mk2(-8388608.0f, -32768.0f), offA23 = mk2(-128.0f, -32768.0f);
    const f2 offB = mk2(-524288.0f, -2048.0f);
    float acc[RS];
#pragma unroll
    for (int r = 0; r < RS; ++r) acc[r] = 0.0f;
    const int ntask = ((nb + 3) >> 2) * kSub;
#pragma unroll 1
    for (int T = warp; T < ntask; T += kKWarps) {
        const int b = (T / kSub) * 4 + bl;
        if (b >= nb) continue;
        const float4* xp = reinterpret_cast<const float4*>(p.x + b * 256 + 64 * j + 16 * (c & 1));
        float4 xa[4], xb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            xa[i] = __ldg(xp + i);
            xb[i] = __ldg(xp + 8 + i);
        }
        f2 xs = mk2(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            xs = add2(xs, add2(mk2(xa[i].x + xa[i].y, xb[i].x + xb[i].y), mk2(xa[i].z + xa[i].w, xb[i].z + xb[i].w)));
        uint4 hd[RS], q[RS];
#pragma unroll
        for (int r = 0; r < RS; ++r) {
            const uint8_t* cp = rowp[r] + static_cast<size_t>(b) * 144;
            q[r] = __ldg(reinterpret_cast<const uint4*>(cp));
            hd[r] = __ldg(reinterpret_cast<const uint4*>(cp - 16 - 16 * c));
        }
#pragma unroll
        for (int r = 0; r < RS; ++r) {
            f2 sa = mk2(0.0f, 0.0f), sb = mk2(0.0f, 0.0f);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = i == 0 ? q[r].x : i == 1 ? q[r].y : i == 2 ? q[r].z : q[r].w;
                const uint32_t v = w >> 16;
                const f2 a01 = add2(mk2u((w & 0xFu) | kMag0, (w & 0xF00u) | kMag8), offA01);
                const f2 a23 = add2(mk2u((w & 0xF0000u) | kMag16, (v & 0xF00u) | kMag8), offA23);
                const f2 b01 = add2(mk2u((w & 0xF0u) | kMag4, (w & 0xF000u) | kMag12), offB);
                const f2 b23 = add2(mk2u((v & 0xF0u) | kMag4, (v & 0xF000u) | kMag12), offB);
                sa = fma2(a01, mk2(xa[i].x, xa[i].y), sa);
                sa = fma2(a23, mk2(xa[i].z, xa[i].w), sa);
                sb = fma2(b01, mk2(xb[i].x, xb[i].y), sb);
                sb = fma2(b23, mk2(xb[i].z, xb[i].w), sb);
            }
            uint32_t sp, mp;
            q4k_pair_scales(hd[r], j, sp, mp);
            const f2 sc = add2(mk2u((sp & 0xFFu) | kMag0, (sp & 0xFF00u) | kMag8), mk2(-8388608.0f, -32768.0f));
            const f2 mn = add2(mk2u((mp & 0xFFu) | kMag0, (mp & 0xFF00u) | kMag8), mk2(-8388608.0f, -32768.0f));
            const float d = f16_bits_to_f32(hd[r].x & 0xFFFFu), dmin = f16_bits_to_f32(hd[r].x >> 16);
            const f2 ds = mul2(mk2(d, d), sc), dm = mul2(mk2(dmin, dmin), mn);
            float a = acc[r];
            a = fmaf(lo(ds), lo(sa) + hi(sa), a);
            a = fmaf(hi(ds), lo(sb) + hi(sb), a);
            a = fmaf(-lo(dm), lo(xs), a);
            a = fmaf(-hi(dm), hi(xs), a);
            acc[r] = a;
        }
    }
    // warp sums into this warp's row subset, then the 8 warps in fixed order
    __shared__ float red[kKWarps][R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int rs = r - sub * RS;
        float v = 0.0f;
#pragma unroll
        for (int t = 0; t < RS; ++t)
            if (t == rs) v = acc[t];
        v = warp_sum(v);
        if (lane == 0) red[warp][r] = v;
    }
    __syncthreads();
    if (warp == 0 && lane < R && row0 + lane < p.N) {
        float out = 0.0f;
#pragma unroll
        for (int w = 0; w < kKWarps; ++w) out += red[w][lane];
        if (p.bias) out += p.bias[row0 + lane];
        if (p.residual) out = p.residual[row0 + lane] + out;
        p.y[row0 + lane] = out;
    }
}

// A 32-bit word of a 2-byte-aligned block: one load when the address is
// 4-byte aligned, two 16-bit loads otherwise (never outside the word).
__device__ __forceinline__ uint32_t ld_word_a2(const uint8_t* a, bool odd) {
    if (!odd) return __ldg(reinterpret_cast<const uint32_t*>(a));
    const unsigned short* h = reinterpret_cast<const unsigned short*>(a);
    return static_cast<uint32_t>(__ldg(h)) | (static_cast<uint32_t>(__ldg(h + 1)) << 16);
}

// Q6_K: lane (rh, h, i0) of a warp task takes positions i0..i0+3 of half h of
// one block, in row half rh of the task's rows: ql words W0 = ql[64h + i0..],
// W1 = ql[64h + 32 + i0..] and qh word H = qh[32h + i0..] hold the 6-bit codes
// of the 16 values 128h + 32k + i0 + e (k, e < 4) as four byte-wise words
//   Q0 = lo(W0) | (H & 3) << 4,  Q1 = lo(W1) | (H >> 2 & 3) << 4,
//   Q2 = hi(W0) | (H >> 4 & 3) << 4,  Q3 = hi(W1) | (H >> 6 & 3) << 4,
// all sharing one int8 scale per k (position group i0 / 16).  Blocks are
// 210 bytes, so consecutive blocks alternate between 4-byte and 2-byte
// alignment; a warp task is ONE block in two rows, which keeps the aligned /
// unaligned load path warp-uniform whenever the row length is a multiple of
// 4 bytes.  Codes become floats with one LOP3 into the mantissa of 2^(23 - p)
// (p = 0, 8, 16; byte 3 after one shift) and a packed subtract of
// 2^(23 - p) + 32.
template <int RS>
__global__ void __launch_bounds__(kKWarps * 32, 3) q6k_matvec_kernel(const KRows p) {
    pdl_launch_dependents();
    constexpr int kSub = kKRows / (2 * RS);   // row subsets; warp w always serves subset w % kSub
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kKRows;
    const int nb = p.K / 256;
    const size_t row_bytes = static_cast<size_t>(nb) * 210;
    // weights before the wait for x, as in the Q4_K kernel
    if (threadIdx.x == 0) prefetch_rows_l2(p.w + row0 * row_bytes, min(kKRows, p.N - row0) * row_bytes);
    pdl_wait();
    const int rh = lane >> 4, h = (lane >> 3) & 1, i0 = 4 * (lane & 7), gsh = 8 * (i0 >> 4);
    const int sub = warp % kSub;
    const uint8_t* rowp[RS];
#pragma unroll
    for (int r = 0; r < RS; ++r)
        rowp[r] = p.w + static_cast<size_t>(min(row0 + sub * 2 * RS + rh * RS + r, p.N - 1)) * row_bytes;
    const f2 off01 = mk2(-8388640.0f, -32800.0f), off23 = mk2(-160.0f, -32800.0f);
    float acc[RS];
#pragma unroll
    for (int r = 0; r < RS; ++r) acc[r] = 0.0f;
    const int ntask = nb * kSub;
#pragma unroll 1
    for (int T = warp; T < ntask; T += kKWarps) {
        const int b = T / kSub;
        const float4* xp = reinterpret_cast<const float4*>(p.x + b * 256 + 128 * h + i0);
        float4 xv[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) xv[k] = __ldg(xp + 8 * k);
#pragma unroll
        for (int r = 0; r < RS; ++r) {
            const uint8_t* blk = rowp[r] + static_cast<size_t>(b) * 210;
            const bool odd = (reinterpret_cast<uintptr_t>(blk) & 2) != 0;
            const uint32_t W0 = ld_word_a2(blk + 64 * h + i0, odd);
            const uint32_t W1 = ld_word_a2(blk + 64 * h + 32 + i0, odd);
            const uint32_t H = ld_word_a2(blk + 128 + 32 * h + i0, odd);
            const unsigned short* s16 = reinterpret_cast<const unsigned short*>(blk + 192 + 8 * h);
            uint32_t su[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) su[k] = static_cast<uint32_t>(__ldg(s16 + k)) >> gsh;
            const float d = f16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(blk + 208)));
            const uint32_t Q[4] = {(W0 & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u),
                                   (W1 & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u),
                                   ((W0 >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u),
                                   ((W1 >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u)};
            // int8 scales as floats: (s ^ 0x80) in the mantissa of 2^23, minus 2^23 + 128
            const f2 sc01 = add2(mk2u((su[0] & 0xFFu) ^ 0x4B000080u, (su[1] & 0xFFu) ^ 0x4B000080u),
                                 mk2(-8388736.0f, -8388736.0f));
            const f2 sc23 = add2(mk2u((su[2] & 0xFFu) ^ 0x4B000080u, (su[3] & 0xFFu) ^ 0x4B000080u),
                                 mk2(-8388736.0f, -8388736.0f));
            const f2 ds01 = mul2(mk2(d, d), sc01), ds23 = mul2(mk2(d, d), sc23);
            float a = acc[r];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t q = Q[k], v = q >> 16;
                const f2 c01 = add2(mk2u((q & 0xFFu) | kMag0, (q & 0xFF00u) | kMag8), off01);
                const f2 c23 = add2(mk2u((q & 0xFF0000u) | kMag16, (v & 0xFF00u) | kMag8), off23);
                const f2 sk = fma2(c23, mk2(xv[k].z, xv[k].w), mul2(c01, mk2(xv[k].x, xv[k].y)));
                const float dk = k == 0 ? lo(ds01) : k == 1 ? hi(ds01) : k == 2 ? lo(ds23) : hi(ds23);
                a = fmaf(dk, lo(sk) + hi(sk), a);
            }
            acc[r] = a;
        }
    }
    // sums over the 16 lanes of each row half, then the 8 warps in fixed order
    __shared__ float red[kKWarps][kKRows];
#pragma unroll
    for (int r = 0; r < kKRows; ++r) {
        const int rs = r - sub * 2 * RS - rh * RS;
        float v = 0.0f;
#pragma unroll
        for (int t = 0; t < RS; ++t)
            if (t == rs) v = acc[t];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
        v += __shfl_xor_sync(0xFFFFFFFFu, v, 16);
        if (lane == 0) red[warp][r] = v;
    }
    __syncthreads();
    if (warp == 0 && lane < kKRows && row0 + lane < p.N) {
        float out = 0.0f;
#pragma unroll
        for (int w = 0; w < kKWarps; ++w) out += red[w][lane];
        if (p.bias) out += p.bias[row0 + lane];
        if (p.residual) out = p.residual[row0 + lane] + out;
        p.y[row0 + lane] = out;
    }
}

// Rows a Q4_K lane walks per task (4, 2 or 1): the choice that finishes the
// CTA's tasks (4 blocks x kKRows / RS each, dealt to 8 warps) in the fewest
// row-block steps, counting a task's x loads as 0.3 of a row.
int q4k_rows_per_lane(int nb) {
    int best = 4, best_cost = 0x7FFFFFFF;
    for (int rs = 4; rs >= 1; rs >>= 1) {
        const int tasks = (nb + 3) / 4 * (kKRows / rs);
        const int cost = (tasks + kKWarps - 1) / kKWarps * (10 * rs + 3);
        if (cost < best_cost) best_cost = cost, best = rs;
    }
    return best;
}

// Rows a Q6_K lane walks per task (2 or 1; a task is one block in 2 RS rows).
int q6k_rows_per_lane(int nb) {
    const int t2 = (nb * (kKRows / 4) + kKWarps - 1) / kKWarps * 23;
    const int t1 = (nb * (kKRows / 2) + kKWarps - 1) / kKWarps * 13;
    return t2 <= t1 ? 2 : 1;
}

}  // namespace

bool matvec_k_supported(int fmt, int K) { return (fmt == FMT_Q4_K || fmt == FMT_Q6_K) && K > 0 && K % 256 == 0; }

cudaError_t launch_matvec_k(int fmt, const MatvecParams& mp, cudaStream_t stream, bool pdl) {
    if (!matvec_k_supported(fmt, mp.K)) return cudaErrorNotSupported;
    if (mp.epilogue != EPI_STORE || mp.norm_out || mp.norm_defer || mp.in_parts || mp.tpl.tp > 1)
        return cudaErrorNotSupported;
    if (reinterpret_cast<uintptr_t>(mp.x) & 15) return cudaErrorNotSupported;
    for (int s = 0; s < mp.nseg; ++s) {
        const MatvecSegment& sg = mp.seg[s];
        if (sg.rows <= 0) continue;
        // Q4_K reads 16-byte header / code vectors, Q6_K 2-byte words
        if (reinterpret_cast<uintptr_t>(sg.w) & (fmt == FMT_Q4_K ? 15 : 1)) return cudaErrorNotSupported;
        KRows p{sg.w, mp.x, sg.y, sg.bias, sg.residual, mp.K, sg.rows};
        cudaLaunchConfig_t cfg = {};
        cfg.blockDim = dim3(kKWarps * 32);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        void (*kern)(const KRows);
        int cta_rows = kKRows;
        if (fmt == FMT_Q4_K && mp.K <= 4096) {
            // short rows: 8-row CTAs, each lane walking 4 rows (x loads shared over 4)
            cta_rows = 8;
            kern = q4k_matvec_kernel<8, 4>;
        } else if (fmt == FMT_Q4_K) {
            const int rs = q4k_rows_per_lane(mp.K / 256);
            kern = rs == 4 ? q4k_matvec_kernel<4, 4> : rs == 2 ? q4k_matvec_kernel<4, 2> : q4k_matvec_kernel<4, 1>;
        } else {
            kern = q6k_rows_per_lane(mp.K / 256) == 2 ? q6k_matvec_kernel<2> : q6k_matvec_kernel<1>;
        }
        cfg.gridDim = dim3((sg.rows + cta_rows - 1) / cta_rows);
        const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace alj
