// Batch-1 GGUF Q4_0, Q8_0, Q4_K and Q6_K dequantise-and-matvec (y = W x) on the integer
// tensor-core path of B200 (sm_100a): mma.sync.m16n8k32 with s8 operands and
// s32 accumulation, for K a multiple of 2048.
//
// Why this shape.  At batch 1 the kernel is HBM-bound only if an SM retires
// ~40 Q4_0 weights per cycle.  The multiply-adds go to the tensor cores; what
// is left on the issue ports is moving and decoding codes, so this kernel is
// built around the fewest instructions per weight:
//   * A operand = the codes themselves.  Q8_0 bytes are s8 as stored (no
//     decode).  A Q4_0 code word gives its eight codes in two LOP3s (plus one
//     shift): (w & 0xF0F0F0F0) ^ 0x80808080 is the four high nibbles as the
//     s8 values 16 (c - 8), and the same on w << 4 gives the low nibbles.
//     Q4_K (GgufQ4RawDot.dotRowQ4K): a 32-byte run of a super-block holds
//     sub-block 2j in its low and 2j + 1 in its high nibbles; quad lanes 0-1
//     take the low, 2-3 the high nibbles of the same bytes, unsigned, and
//     each row adds d scale 2^-F (digits) - dmin min sum(x) per sub-block.
//     Q6_K (GgufQ6RawDot.dotRowQ6K): the 6-bit codes (ql nibble | qh bits)
//     as u8 of one 32-value block per MMA, quad lanes 0-1 / 2-3 its two
//     16-value scale groups; the -32 offset enters as -32 sum(x) per group.
//   * B operand = x, split exactly into three balanced int8 digits per
//     32-element block: X = rint(x 2^F) with F chosen from the block's max
//     |x| so that |X| <= 2^22, X = h 2^16 + m 2^8 + l, l, m in [-128, 127],
//     h in [-64, 64].  One MMA column per digit, so every product and every
//     partial sum is an exact integer (|sum| < 2^19 per column): the tensor
//     core rounds nothing.  The block value d 2^-F (h 2^16 + m 2^8 + l) is
//     formed in fp32 once per block, which is the only rounding besides the
//     fp32 sums over blocks.  x keeps 22 bits relative to its block maximum.
//   * One k32 MMA covers two blocks of 16 rows: k-slots of quad lanes 0-1
//     carry the even block of a block pair, lanes 2-3 the odd block, and
//     columns 0-2 / 4-6 hold the digits of the even / odd block.  So every
//     lane's accumulator columns belong to one block and one fp16 scale.
//
// Data flow per CTA (one CTA per SM; 16 consumer warps, a TMA producer warp
// and an epilogue warp; up to 8 stages of ~18 KB in flight):
//   * rows are dealt out in balanced units of 4 and walked in slabs of <= 16
//     rows (a slab never straddles a weight segment) x chunks of 2048 (Q4_0)
//     or 1024 (Q8_0) columns;
//   * the producer copies each slab-chunk with 2-D TMA boxes of 8 or 4 rows
//     whose inner extent is the chunk plus 16 bytes: smem rows are padded by
//     16 bytes (a 4- or 20-word bank shift per row), which makes every
//     fragment load of a quad (four distinct words mod 4) conflict-free;
//   * warp w owns a fixed run of block pairs in every chunk (2 for Q4_0, 1
//     for Q8_0), converts their x into B-fragment records once per launch
//     (read by no other warp), and for each stage loads its code words, runs
//     two MMAs per block pair and folds d 2^-F per block into fp32 row sums;
//   * per-warp row sums go through a shared-memory ring to the epilogue
//     warp, which adds them in fixed warp order (bit-identical repeat calls)
//     and applies bias / residual.
// Every mbarrier wait is bounded (ALJ_FAULT_TIMEOUT in the device fault word).
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

namespace alj {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();   // matvec.cu

namespace {

constexpr int kCW = 16;                      // consumer warps
constexpr int kProducerWarp = kCW;
constexpr int kEpilogueWarp = kCW + 1;
constexpr int kThreads = (kCW + 2) * 32;
constexpr int kUnit = 4;                     // rows per balancing unit
constexpr int kMaxStages = 8;
constexpr int kRing = 4;                     // slab partial buffers
constexpr int kRecBytes = 208;               // B fragments of one block pair: 12 active lanes x 16 B + a zero slot
constexpr int kZeroSlot = 12;                // the slot that lanes with no B operand read
constexpr int kSlabUnits = 8;                // a slab is 32 rows (two 16-row MMA tiles) ...
constexpr int kMaxSlabUnits = 9;             // ... or 36 when it absorbs a CTA's one leftover unit
constexpr int kStageRows = 36;               // stage capacity (a third tile's reads of rows 36..39 fall
                                             // into the next stage or the records: garbage rows, never stored)
constexpr int kRedRows = kUnit * kMaxSlabUnits;
constexpr int kSmemMax = 232448;             // 227 KB opt-in per CTA
constexpr uint32_t kMagic = 0x4B400000u;     // bits of 1.5 * 2^23: fma(x, s, magic) = magic + rint(x s)

template <int FMT>
struct IFmt;
template <>
struct IFmt<FMT_Q4_0> {
    static constexpr int kPairBytes = 36;    // two 18-byte blocks
    static constexpr int kChunkPairs = 32;   // 2048 columns
    static constexpr int kChunkBytes = 1152;
    static constexpr int kRowPad = 16;       // a 4-word bank shift per row
    static constexpr int kWordsPerRow = 2;   // code words a lane decodes per row and pair
};
template <>
struct IFmt<FMT_Q8_0> {
    static constexpr int kPairBytes = 68;    // two 34-byte blocks
    static constexpr int kChunkPairs = 16;   // 1024 columns
    static constexpr int kChunkBytes = 1088;
    static constexpr int kRowPad = 16;
    static constexpr int kWordsPerRow = 4;
};
// Q4_K: a "pair" is the 64 values of one 32-byte code run of a 144-byte
// super-block (sub-blocks 2j and 2j + 1: low and high nibbles of the same
// bytes); a warp's two pairs are the adjacent runs 2(w & 1), 2(w & 1) + 1 of
// super-block w / 2 of the chunk, 32 bytes apart.
template <>
struct IFmt<FMT_Q4_K> {
    static constexpr int kPairBytes = 32;    // step between a warp's two code runs
    static constexpr int kChunkPairs = 32;   // 2048 columns = 8 super-blocks
    static constexpr int kChunkBytes = 1152;
    // an 8-word bank shift per row: the 16-byte code loads of a quarter warp
    // (rows g, g + 1, both 16-byte halves of a run) hit four distinct groups
    static constexpr int kRowPad = 32;
    static constexpr int kWordsPerRow = 4;   // a lane takes one nibble of 16 code bytes per row and pair
};
// Q6_K: 210-byte super-blocks (ql[128] low nibbles, qh[64] two high bits,
// int8 scales[16] per 16 values, fp16 d), 8 per 2048-column chunk (1680
// bytes).  A "pair" is 64 values = blocks k0, k0 + 1 (k0 = 2 (j % 2)) of
// half h = j / 2 of a super-block; a warp's two pairs (j = 2 (w % 2) and
// + 1, super-block w / 2) read the same ql / qh bytes (other nibble, other
// bit pair).  Super-blocks are only 2-byte aligned in shared memory.
template <>
struct IFmt<FMT_Q6_K> {
    static constexpr int kPairBytes = 0;     // the warp's two pairs share their code bytes
    static constexpr int kChunkPairs = 32;   // 2048 columns = 8 super-blocks
    static constexpr int kChunkBytes = 1680;
    static constexpr int kRowPad = 16;
    static constexpr int kWordsPerRow = 0;
};
template <int FMT>
struct IGeom {
    static constexpr int kChunkCols = IFmt<FMT>::kChunkPairs * 64;
    static constexpr int kChunkBytes = IFmt<FMT>::kChunkBytes;   // 1152 | 1088 | 1152
    static constexpr int kRowStride = kChunkBytes + IFmt<FMT>::kRowPad;                  // 1168 | 1104 | 1184
    static constexpr int kBoxElems = kRowStride / 8;                                     // uint64 elements
    // TMA destinations (stage base + 8-row box offsets) must be 128-byte aligned
    static constexpr int kStageBytes = (kStageRows * kRowStride + 127) / 128 * 128;
    static_assert((8 * kRowStride) % 128 == 0, "8-row box offsets must stay 128-byte aligned");
    static_assert(kStageBytes % 128 == 0, "stage bases must stay 128-byte aligned");
    static constexpr int kPairsPerWarp = IFmt<FMT>::kChunkPairs / kCW;                   // 2 | 1
};

// Source word (index into the pair's 32-bit words) of code word `w` of quad
// lane t.  -1 marks the word the even block splits across its scale words:
// bytes 2-3 of word 0 and bytes 0-1 of word 4 (Q4_0) or word 8 (Q8_0).
// Quad lanes 0-1 take the even block's code bytes, lanes 2-3 the odd block's;
// each load instruction of a quad reads four words that are distinct mod 4.
__host__ __device__ constexpr int src_word(int fmt, int t, int w) {
    return fmt == FMT_Q4_0 ? (t == 0 ? (w == 0 ? 1 : 2) : t == 1 ? (w == 0 ? 3 : -1) : t == 2 ? (w == 0 ? 8 : 5)
                                                                                                : (w == 0 ? 6 : 7))
                           : (t == 0 ? 1 + 2 * w
                              : t == 1 ? (w < 3 ? 2 + 2 * w : -1)
                              : t == 2 ? (w == 0 ? 11 : w == 1 ? 9 : w == 2 ? 15 : 13)
                                       : (w == 0 ? 12 : w == 1 ? 10 : w == 2 ? 16 : 14));
}
// Byte of the pair that byte q of lane t's code word w holds.
__host__ __device__ constexpr int word_byte(int fmt, int t, int w, int q) {
    return src_word(fmt, t, w) >= 0 ? 4 * src_word(fmt, t, w) + q
                                    : (q < 2 ? 2 + q : (fmt == FMT_Q4_0 ? 14 : 30) + q);
}
// Block element (0..31, within the lane's block) multiplied at k-slot byte q
// of operand register r (0 = a0/a1, 1 = a2/a3) in MMA m of a block pair.
// Q4_K: quad lanes 0-1 take the low nibbles (sub-block 2j), lanes 2-3 the
// high nibbles (sub-block 2j + 1) of the same 16 bytes per lane: byte
// 16 (t % 2) + 4 w + q of the run holds element 16 (t % 2) + 4 w + q of
// both, and code word w = 2 m + r feeds operand r of MMA m.
// Q6_K (pair-relative): MMA m is block m of the pair, quad lanes 0-1 its
// values 0..15, lanes 2-3 values 16..31, 8 per lane.
__host__ __device__ constexpr int slot_elem(int fmt, int t, int m, int r, int q) {
    return fmt == FMT_Q6_K   ? 32 * m + 16 * (t >> 1) + 8 * (t & 1) + 4 * r + q
           : fmt == FMT_Q4_K ? 16 * (t & 1) + 4 * (2 * m + r) + q
           : fmt == FMT_Q4_0 ? (word_byte(fmt, t, r, q) - (t < 2 ? 2 : 20)) + 16 * m
                             : (word_byte(fmt, t, 2 * m + r, q) - (t < 2 ? 2 : 36));
}

struct alignas(64) ImmaSegment {
    CUtensorMap map8;                        // box {row chunk + 16 B, 8 rows}
    CUtensorMap map4;                        // box {row chunk + 16 B, 4 rows}
    const float* bias;
    const float* residual;
    float* y;
    int rows;
    int row0;
};

struct alignas(64) ImmaParams {
    ImmaSegment seg[3];
    int nseg;
    int K;
    int total_rows;
    const float* x;
    const uint8_t* prefetch;
    size_t prefetch_bytes;
    // deferred RMSNorm (decode step, one segment): the epilogue also stores
    // norm_out = y * norm_w and this CTA's sum of y^2 in norm_partials[cta];
    // a launch with in_parts scales x by 1 / sqrt(sum(in_parts) / in_rows +
    // in_eps) as it converts it
    float* norm_out;
    const float* norm_w;
    float* norm_partials;
    const float* in_parts;
    int in_nparts;
    int in_rows;
    float in_eps;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
// High nibbles as s8 16 (c - 8); the same on (w << 4) gives the low nibbles.
__device__ __forceinline__ uint32_t nib_s8(uint32_t w) { return lop3_and_xor(w, 0xF0F0F0F0u, 0x80808080u); }

// Slabs of 32 rows of a CTA's unit range, split at segment boundaries; a
// single unit left over at the end joins the last slab (36 rows), so CTAs
// that hold one unit more than others walk the same number of stages.
struct SlabWalk {
    int u, u_end;
    __device__ __forceinline__ bool next(const ImmaParams& p, int& seg, int& su, int& nunits) {
        if (u >= u_end) return false;
        seg = 0;
        if (p.nseg > 1 && u * kUnit >= p.seg[1].row0) seg = 1;
        if (p.nseg > 2 && u * kUnit >= p.seg[2].row0) seg = 2;
        const int seg_end = (p.seg[seg].row0 + p.seg[seg].rows) / kUnit;
        su = u;
        const int avail = min(u_end, seg_end) - u;
        nunits = avail == kSlabUnits + 1 ? avail : min(kSlabUnits, avail);
        u += nunits;
        return true;
    }
};

// Shared-memory loads at a 32-bit address plus a compile-time byte offset
// (folded into the instruction).
template <int OFF>
__device__ __forceinline__ uint32_t lds_at(uint32_t a) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ uint4 lds4_at(uint32_t a) {
    uint4 v;
    asm("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4+%5];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "r"(a), "n"(OFF));
    return v;
}

// Per-lane constants of the consumer loop (lane (g, t) of the MMA).
struct LaneCtx {
    uint32_t woff[4];     // smem byte offsets of this lane's code words in row g, pair 0 of the warp
    uint32_t v0, vd;      // the pair's word 0 (even block's d) and the word holding the odd block's d
    uint32_t sel_fix;     // PRMT joining the even block's split code word (lane 1)
    uint32_t sel_d;       // PRMT picking this lane's block scale
    uint32_t brec;        // smem address of this lane's B record slot, block pair 0
    uint32_t xsl;         // smem address of this lane's block scale 2^-F, block pair 0
    f2 kd0, kd1;          // digit weights of accumulator columns 2t, 2t + 1
    // Q4_K only
    uint32_t nmask;       // 0x0F0F0F0F: this lane's sub-block is the low nibbles, 0xF0F0F0F0: the high ones
    uint32_t oddw;        // the warp's runs are sub-blocks 4..7 of their super-block
    uint32_t ksel[2];     // PRMT gathering the (scale, min) bytes of the lane's sub-block, run J
    uint32_t xsum_off;    // bytes from a block scale to the block's sum of x
    float kmin;           // 1 on the quad lane that adds its sub-block's min term (Q6_K: offset term), else 0
    // Q6_K only (oddw: the warp's super-block starts 2 bytes off a word)
    uint32_t qoff[3];     // word-aligned offsets (row g, tile 0) of the lane's ql bytes (blocks 0, 1) and qh bytes
    uint32_t soff;        // word-aligned offset of the word holding the lane's first scale byte
    uint32_t ssel[4];     // sign-extending PRMT of scale e = 2 J + m out of words (0, 1), or (1, 2) if bit e of sw
    uint32_t sw;
    uint32_t doff, dsh;   // d's word-aligned offset and bit position (0 or 16)
    uint32_t xs16l;       // smem address of this lane's half sums of x (its half of block 0), pair 0
};

__device__ __forceinline__ float f16_lo(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFFu)));
}
__device__ __forceinline__ float f16_hi(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16)));
}
// 6-bit scale and min of the lane's sub-block s (GGUF's packed 12 bytes q in
// header words h.y, h.z, h.w): s < 4: q[s] & 63, q[s + 4] & 63; s >= 4:
// (q[s + 4] & 15) | (q[s - 4] >> 6) << 4, (q[s + 4] >> 4) | (q[s] >> 6) << 4.
__device__ __forceinline__ void k_scale_min(const LaneCtx& L, uint32_t sel, const uint4& h, float& sc, float& mn) {
    if (L.oddw) {
        const uint32_t v = prmt(h.y, h.w, sel);         // byte 0 = q[s - 4], byte 1 = q[s + 4]
        const uint32_t v2 = prmt(h.z, h.z, sel & 0xFu);  // byte 0 = q[s]
        sc = static_cast<float>(((v >> 8) & 15u) | ((v >> 2) & 0x30u));
        mn = static_cast<float>(((v >> 12) & 15u) | ((v2 >> 2) & 0x30u));
    } else {
        const uint32_t v = prmt(h.y, h.z, sel);         // byte 0 = q[s], byte 1 = q[s + 4]
        sc = static_cast<float>(v & 63u);
        mn = static_cast<float>((v >> 8) & 63u);
    }
}

// One 16-row tile (RT) of block pair J of a stage: 2 MMAs and the fp32 fold.
// st[w] = stage base + woff[w]; every offset below is a compile-time constant.
template <int FMT, int J, int RT>
__device__ __forceinline__ void pair_tile(const LaneCtx& L, const uint32_t (&st)[4], uint32_t sv0, uint32_t svd,
                                          const uint4& B, const f2& xs2, f2& y) {
    constexpr int kRS = IGeom<FMT>::kRowStride;
    constexpr int kNW = IFmt<FMT>::kWordsPerRow;
    constexpr int O = RT * 16 * kRS + J * IFmt<FMT>::kPairBytes;
    constexpr int O8 = RT < 2 ? O + 8 * kRS : O;       // row g + 8 (tile 2: rows 32..35 only)
    uint32_t W0[kNW], W1[kNW];
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
        W0[w] = lds_at<O>(st[w]);
        W1[w] = lds_at<O8>(st[w]);
    }
    const uint32_t v00 = lds_at<O>(sv0), v01 = lds_at<O8>(sv0);
    const uint32_t vd0 = lds_at<O>(svd), vd1 = lds_at<O8>(svd);
    W0[kNW - 1] = prmt(W0[kNW - 1], v00, L.sel_fix);
    W1[kNW - 1] = prmt(W1[kNW - 1], v01, L.sel_fix);
    const uint32_t d0 = prmt(v00, vd0, L.sel_d), d1 = prmt(v01, vd1, L.sel_d);
    int acc[4] = {0, 0, 0, 0};
    if constexpr (FMT == FMT_Q4_0) {
        imma(acc, nib_s8(W0[0] << 4), nib_s8(W1[0] << 4), nib_s8(W0[1] << 4), nib_s8(W1[1] << 4), B.x, B.y);
        imma(acc, nib_s8(W0[0]), nib_s8(W1[0]), nib_s8(W0[1]), nib_s8(W1[1]), B.z, B.w);
    } else {
        imma(acc, W0[0], W1[0], W0[1], W1[1], B.x, B.y);
        imma(acc, W0[2], W1[2], W0[3], W1[3], B.z, B.w);
    }
    const f2 dd = mk2(__half2float(__ushort_as_half(static_cast<unsigned short>(d0 & 0xFFFFu))),
                      __half2float(__ushort_as_half(static_cast<unsigned short>(d1 & 0xFFFFu))));
    const f2 c0 = mk2(static_cast<float>(acc[0]), static_cast<float>(acc[2]));
    const f2 c1 = mk2(static_cast<float>(acc[1]), static_cast<float>(acc[3]));
    y = fma2(mul2(dd, xs2), fma2(c1, L.kd1, mul2(c0, L.kd0)), y);
}

// Q4_K, one 16-row tile RT of a warp's stage work: the super-block header of
// rows g and g + 8 is read and its d / dmin decoded once for both code runs
// J; per run, the lane's 16 code bytes per row (one 16-byte load each; rows
// are 1184 bytes apart, so a quarter warp's four addresses hit distinct
// 16-byte bank groups), one AND keeps its nibbles -- c (low) or 16 c (high,
// within u8) -- and two u8 x s8 MMAs give the sub-block dot; per row
// d * scale * 2^-F * (digits) - dmin * min * sum(x), the min once per quad.
__device__ __forceinline__ void immau(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <int RT>
__device__ __forceinline__ void tile_k(const LaneCtx& L, uint32_t sc0, uint32_t sh, const uint4 (&B)[2],
                                       const f2 (&xs2)[2], const f2 (&xm2)[2], f2& y) {
    constexpr int kRS = IGeom<FMT_Q4_K>::kRowStride;
    constexpr int H = RT * 16 * kRS;                    // row g of the tile
    constexpr int H8 = RT < 2 ? H + 8 * kRS : H;        // row g + 8 (tile 2: rows 32..35 only)
    const uint4 h0 = lds4_at<H>(sh), h1 = lds4_at<H8>(sh);
    const f2 dv = mk2(f16_lo(h0.x), f16_lo(h1.x));
    const f2 dmv = mk2(f16_hi(h0.x), f16_hi(h1.x));
#pragma unroll
    for (int J = 0; J < 2; ++J) {
        constexpr int kPB = IFmt<FMT_Q4_K>::kPairBytes;
        const uint4 q0 = J == 0 ? lds4_at<H>(sc0) : lds4_at<H + kPB>(sc0);
        const uint4 q1 = J == 0 ? lds4_at<H8>(sc0) : lds4_at<H8 + kPB>(sc0);
        int acc[4] = {0, 0, 0, 0};
        immau(acc, q0.x & L.nmask, q1.x & L.nmask, q0.y & L.nmask, q1.y & L.nmask, B[J].x, B[J].y);
        immau(acc, q0.z & L.nmask, q1.z & L.nmask, q0.w & L.nmask, q1.w & L.nmask, B[J].z, B[J].w);
        float s0, m0, s1, m1;
        k_scale_min(L, L.ksel[J], h0, s0, m0);
        k_scale_min(L, L.ksel[J], h1, s1, m1);
        const f2 dd = mul2(dv, mk2(s0, s1));
        const f2 mm = mul2(dmv, mk2(m0, m1));
        const f2 c0 = mk2(static_cast<float>(acc[0]), static_cast<float>(acc[2]));
        const f2 c1 = mk2(static_cast<float>(acc[1]), static_cast<float>(acc[3]));
        y = fma2(mul2(dd, xs2[J]), fma2(c1, L.kd1, mul2(c0, L.kd0)), y);
        y = fma2(mm, xm2[J], y);
    }
}
template <int NRT>
__device__ __forceinline__ void stage_pairs_k(const LaneCtx& L, uint32_t sc0, uint32_t sh, uint32_t pb, uint32_t px,
                                              f2& y0, f2& y1, f2& y2) {
    const uint4 B[2] = {lds4_at<0>(pb), lds4_at<kRecBytes>(pb)};
    const float xa = __uint_as_float(lds_at<0>(px)), xb = __uint_as_float(lds_at<8>(px));
    const float ma = -L.kmin * __uint_as_float(lds_at<0>(px + L.xsum_off));
    const float mb = -L.kmin * __uint_as_float(lds_at<8>(px + L.xsum_off));
    const f2 xs2[2] = {mk2(xa, xa), mk2(xb, xb)};
    const f2 xm2[2] = {mk2(ma, ma), mk2(mb, mb)};
    tile_k<0>(L, sc0, sh, B, xs2, xm2, y0);
    if constexpr (NRT >= 2) tile_k<1>(L, sc0, sh, B, xs2, xm2, y1);
    if constexpr (NRT >= 3) tile_k<2>(L, sc0, sh, B, xs2, xm2, y2);
}

// Q6_K: 8 bytes at row offset O + a (a word-aligned; `mis`: the field starts
// 2 bytes past a), as two words.
template <int O>
__device__ __forceinline__ uint2 q6_field(uint32_t a, uint32_t mis) {
    const uint32_t w0 = lds_at<O>(a), w1 = lds_at<O + 4>(a);
    if (!mis) return make_uint2(w0, w1);
    const uint32_t w2 = lds_at<O + 8>(a);
    return make_uint2(__funnelshift_r(w0, w1, 16), __funnelshift_r(w1, w2, 16));
}
// Scale e = 2 J + m of the lane's half (int8, sign-extended by PRMT).
__device__ __forceinline__ float q6_scale(const LaneCtx& L, int e, uint32_t s0, uint32_t s1, uint32_t s2) {
    const bool hw = (L.sw >> e) & 1u;
    return static_cast<float>(static_cast<int>(prmt(hw ? s1 : s0, hw ? s2 : s1, L.ssel[e])));
}
// 6-bit codes of 4 values: ql nibble J, qh bits 2k..2k+1 (k = 2 J + m) on top.
template <int J, int M>
__device__ __forceinline__ uint32_t q6_codes(uint32_t ql, uint32_t qh) {
    constexpr int k = 2 * J + M;
    const uint32_t lo = (J == 0 ? ql : ql >> 4) & 0x0F0F0F0Fu;
    const uint32_t hi = (k == 0 ? qh << 4 : k == 1 ? qh << 2 : k == 2 ? qh : qh >> 2) & 0x30303030u;
    return lo | hi;
}
// Q6_K, one 16-row tile RT: per row the lane's ql (blocks 0, 1) and qh bytes,
// its four scales and d, shared by the warp's two pairs J; per (J, block m)
// one u8 x s8 MMA on the codes q in 0..63, then per row
// d * scale * (2^-F (digits) - 32 sum(x of the half)), the offset term once
// per quad.
template <int RT>
__device__ __forceinline__ void tile_q6(const LaneCtx& L, uint32_t sb, const uint4 (&B)[2], const f2 (&xs2)[2][2],
                                        const f2 (&xm2)[2][2], f2& y) {
    constexpr int kRS = IGeom<FMT_Q6_K>::kRowStride;
    constexpr int R0 = RT * 16 * kRS;
    constexpr int R8 = RT < 2 ? R0 + 8 * kRS : R0;      // row g + 8 (tile 2: rows 32..35 only)
    const uint2 ql0[2] = {q6_field<R0>(sb + L.qoff[0], L.oddw), q6_field<R8>(sb + L.qoff[0], L.oddw)};
    const uint2 ql1[2] = {q6_field<R0>(sb + L.qoff[1], L.oddw), q6_field<R8>(sb + L.qoff[1], L.oddw)};
    const uint2 qh[2] = {q6_field<R0>(sb + L.qoff[2], L.oddw), q6_field<R8>(sb + L.qoff[2], L.oddw)};
    const uint32_t sa = sb + L.soff, da = sb + L.doff;
    const uint32_t s00 = lds_at<R0>(sa), s01 = lds_at<R0 + 4>(sa), s02 = lds_at<R0 + 8>(sa);
    const uint32_t s10 = lds_at<R8>(sa), s11 = lds_at<R8 + 4>(sa), s12 = lds_at<R8 + 8>(sa);
    const float d0 = __half2float(__ushort_as_half(static_cast<unsigned short>((lds_at<R0>(da) >> L.dsh) & 0xFFFFu)));
    const float d1 = __half2float(__ushort_as_half(static_cast<unsigned short>((lds_at<R8>(da) >> L.dsh) & 0xFFFFu)));
#pragma unroll
    for (int J = 0; J < 2; ++J)
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const uint2 lo0 = m == 0 ? ql0[0] : ql1[0], lo1 = m == 0 ? ql0[1] : ql1[1];
            uint32_t a0, a1, a2, a3;
            if (J == 0 && m == 0) {
                a0 = q6_codes<0, 0>(lo0.x, qh[0].x); a1 = q6_codes<0, 0>(lo1.x, qh[1].x);
                a2 = q6_codes<0, 0>(lo0.y, qh[0].y); a3 = q6_codes<0, 0>(lo1.y, qh[1].y);
            } else if (J == 0) {
                a0 = q6_codes<0, 1>(lo0.x, qh[0].x); a1 = q6_codes<0, 1>(lo1.x, qh[1].x);
                a2 = q6_codes<0, 1>(lo0.y, qh[0].y); a3 = q6_codes<0, 1>(lo1.y, qh[1].y);
            } else if (m == 0) {
                a0 = q6_codes<1, 0>(lo0.x, qh[0].x); a1 = q6_codes<1, 0>(lo1.x, qh[1].x);
                a2 = q6_codes<1, 0>(lo0.y, qh[0].y); a3 = q6_codes<1, 0>(lo1.y, qh[1].y);
            } else {
                a0 = q6_codes<1, 1>(lo0.x, qh[0].x); a1 = q6_codes<1, 1>(lo1.x, qh[1].x);
                a2 = q6_codes<1, 1>(lo0.y, qh[0].y); a3 = q6_codes<1, 1>(lo1.y, qh[1].y);
            }
            int acc[4] = {0, 0, 0, 0};
            immau(acc, a0, a1, a2, a3, m == 0 ? B[J].x : B[J].z, m == 0 ? B[J].y : B[J].w);
            const int e = 2 * J + m;
            const f2 dd = mk2(d0 * q6_scale(L, e, s00, s01, s02), d1 * q6_scale(L, e, s10, s11, s12));
            const f2 c0 = mk2(static_cast<float>(acc[0]), static_cast<float>(acc[2]));
            const f2 c1 = mk2(static_cast<float>(acc[1]), static_cast<float>(acc[3]));
            y = fma2(dd, fma2(xs2[J][m], fma2(c1, L.kd1, mul2(c0, L.kd0)), xm2[J][m]), y);
        }
}
template <int NRT>
__device__ __forceinline__ void stage_pairs_q6(const LaneCtx& L, uint32_t sb, uint32_t pb, uint32_t px, uint32_t px16,
                                               f2& y0, f2& y1, f2& y2) {
    const uint4 B[2] = {lds4_at<0>(pb), lds4_at<kRecBytes>(pb)};
    f2 xs2[2][2], xm2[2][2];
#pragma unroll
    for (int J = 0; J < 2; ++J)
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const float xs = __uint_as_float(J == 0 ? (m == 0 ? lds_at<0>(px) : lds_at<4>(px))
                                                    : (m == 0 ? lds_at<8>(px) : lds_at<12>(px)));
            const float hs = __uint_as_float(J == 0 ? (m == 0 ? lds_at<0>(px16) : lds_at<8>(px16))
                                                    : (m == 0 ? lds_at<16>(px16) : lds_at<24>(px16)));
            xs2[J][m] = mk2(xs, xs);
            const float xm = -32.0f * L.kmin * hs;
            xm2[J][m] = mk2(xm, xm);
        }
    tile_q6<0>(L, sb, B, xs2, xm2, y0);
    if constexpr (NRT >= 2) tile_q6<1>(L, sb, B, xs2, xm2, y1);
    if constexpr (NRT >= 3) tile_q6<2>(L, sb, B, xs2, xm2, y2);
}

// All of a stage's work for one warp: kPPW block pairs x NRT row tiles.
template <int FMT, int NRT, int J = 0>
__device__ __forceinline__ void stage_pairs(const LaneCtx& L, const uint32_t (&st)[4], uint32_t sv0, uint32_t svd,
                                            uint32_t pb, uint32_t px, f2& y0, f2& y1, f2& y2) {
    constexpr int kRecBytesT = kRecBytes;
    const uint4 B = lds4_at<J * kRecBytesT>(pb);
    const float xsv = __uint_as_float(lds_at<J * 8>(px));
    const f2 xs2 = mk2(xsv, xsv);
    pair_tile<FMT, J, 0>(L, st, sv0, svd, B, xs2, y0);
    if constexpr (NRT >= 2) pair_tile<FMT, J, 1>(L, st, sv0, svd, B, xs2, y1);
    if constexpr (NRT >= 3) pair_tile<FMT, J, 2>(L, st, sv0, svd, B, xs2, y2);
    if constexpr (J + 1 < IGeom<FMT>::kPairsPerWarp)
        stage_pairs<FMT, NRT, J + 1>(L, st, sv0, svd, pb, px, y0, y1, y2);
}

// x digits of every block pair this warp owns (its run of kPPW pairs in each
// chunk) into B-fragment records and per-block scales, in units of two
// pairs.  The x loads of up to kXBatch units go out together (every CTA reads
// all of x, so those lines are contended in L2: one round trip per batch).
//   pass A: lane l holds x[4 (l % 16) ..] of unit pair j = l / 16; 8-lane
//           groups form each block's max |x| and scale 2^F; each lane writes
//           the three digit bytes of its four elements, in element order,
//           into the warp's scratch (one word per digit);
//   pass B: lane (pair j, group (t, m, r)) gathers the four digit bytes that
//           k-slot bytes 0..3 of operand r of MMA m carry for quad lane t
//           (two words and a PRMT per digit) and writes the three record
//           words of lanes (g, t), g = digit (t < 2) or 4 + digit (t >= 2).
constexpr int kXBatch = 8;
constexpr int kScratchBytes = 2 * 3 * 128;  // per warp: digit planes h, m, l of two units' 128 elements

template <int FMT>
__device__ __forceinline__ int unit_pair(int u, int j, int warp) {
    constexpr int kPPW = IGeom<FMT>::kPairsPerWarp;
    constexpr int kCP = IFmt<FMT>::kChunkPairs;
    return kPPW == 2 ? u * kCP + warp * 2 + j : (2 * u + j) * kCP + warp;
}

// Pass A for one unit: lane l's four elements of unit pair l / 16 into the
// three digit-plane words of `scratch`, and the block scales.
template <int FMT>
__device__ __forceinline__ void stage_pass_a(const float4& v, int u, int warp, int lane, float* xs, uint32_t* swr,
                                             float* xsum) {
    float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    // exponent field E of the max: scale 2^F, F = 148 - E (max 2^F in
    // [2^21, 2^22)); E clamped below so that 2^-F / 16 stays normal;
    // a block holding Inf or NaN gets a NaN scale (its rows become NaN).
    const uint32_t eb = (__float_as_uint(mx) >> 23) & 0xFFu;
    const uint32_t ec = eb < 26u ? 26u : eb;
    const float sc = eb == 0xFFu ? 0.0f : __uint_as_float((275u - ec) << 23);
    const float inv = eb == 0xFFu ? __uint_as_float(0x7FC00000u)
                                  : __uint_as_float((ec - 21u - (FMT == FMT_Q4_0 ? 4u : 0u)) << 23);
    if ((lane & 7) == 0) xs[2 * unit_pair<FMT>(u, lane >> 4, warp) + ((lane >> 3) & 1)] = inv;
    if constexpr (FMT == FMT_Q6_K) {   // each 16-value half's sum of x, for the -32 offset
        float sm = (v.x + v.y) + (v.z + v.w);
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        if ((lane & 3) == 0) xsum[4 * unit_pair<FMT>(u, lane >> 4, warp) + ((lane >> 2) & 3)] = sm;
    }
    if constexpr (FMT == FMT_Q4_K) {   // the block's sum of x, for the min term
        float sm = (v.x + v.y) + (v.z + v.w);
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        sm += __shfl_xor_sync(0xffffffffu, sm, 4);
        if ((lane & 7) == 0) xsum[2 * unit_pair<FMT>(u, lane >> 4, warp) + ((lane >> 3) & 1)] = sm;
    }
    const float xv[4] = {v.x, v.y, v.z, v.w};
    uint32_t bits[4], mid[4], hig[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        bits[q] = __float_as_uint(__fmaf_rn(xv[q], sc, __uint_as_float(kMagic)));   // magic + X
        mid[q] = bits[q] + 0x80u;                 // byte 1 = m digit of X
        hig[q] = bits[q] - 0x3F7F80u;             // byte 2 = h digit of X
    }
    swr[0 * 32 + lane] = prmt(prmt(hig[0], hig[1], 0x0062u), prmt(hig[2], hig[3], 0x6200u), 0x7610u);
    swr[1 * 32 + lane] = prmt(prmt(mid[0], mid[1], 0x0051u), prmt(mid[2], mid[3], 0x5100u), 0x7610u);
    swr[2 * 32 + lane] = prmt(prmt(bits[0], bits[1], 0x0040u), prmt(bits[2], bits[3], 0x4000u), 0x7610u);
}

template <int FMT>
__device__ __forceinline__ void stage_x(const float* __restrict__ x, int nunits, uint8_t* rec, float* xs,
                                        uint8_t* scratch, int warp, int lane, float* xsum, float in_s) {
    const int jb = lane >> 4, gi = lane & 15;                  // pass B: (pair, t, m, r)
    const int t = gi >> 2, m = (gi >> 1) & 1, r = gi & 1;
    const int e0 = slot_elem(FMT, t, m, r, 0), e2 = slot_elem(FMT, t, m, r, 2);
    const int bbase = jb * 64 + (FMT != FMT_Q6_K && t >= 2 ? 32 : 0);   // Q6_K's slots are pair-relative
    const int wa = (bbase + e0) >> 2, wb = (bbase + e2) >> 2;  // scratch words holding bytes e0, e0+1 / e2, e2+1
    const uint32_t gsel = static_cast<uint32_t>((e0 & 3) | ((e0 & 3) + 1) << 4 | (4 + (e2 & 3)) << 8 |
                                                (5 + (e2 & 3)) << 12);
    uint32_t* sw = reinterpret_cast<uint32_t*>(scratch);      // two units: [2][3 planes][32 words]
    // pass B of one unit from scratch half h
    auto pass_b = [&](int u, int h) {
        const uint32_t* s = sw + h * 96;
        uint8_t* prec = rec + static_cast<size_t>(unit_pair<FMT>(u, jb, warp)) * kRecBytes;
        uint8_t* slot = prec + (t < 2 ? t : 4 + t) * 16 + 4 * (2 * m + r);
#pragma unroll
        for (int d = 0; d < 3; ++d)
            *reinterpret_cast<uint32_t*>(slot + 32 * d) = prmt(s[d * 32 + wa], s[d * 32 + wb], gsel);
        if (gi < 4) reinterpret_cast<uint32_t*>(prec + kZeroSlot * 16)[gi] = 0u;
    };
    for (int u0 = 0; u0 < nunits; u0 += kXBatch) {
        float4 v[kXBatch];
#pragma unroll
        for (int b = 0; b < kXBatch; ++b)
            if (u0 + b < nunits)
                v[b] = __ldg(reinterpret_cast<const float4*>(x + static_cast<size_t>(unit_pair<FMT>(u0 + b, lane >> 4, warp)) * 64) +
                             (lane & 15));
        if (in_s != 1.0f) {
#pragma unroll
            for (int b = 0; b < kXBatch; ++b) {
                v[b].x *= in_s;
                v[b].y *= in_s;
                v[b].z *= in_s;
                v[b].w *= in_s;
            }
        }
        // two units per round: their shuffle / PRMT chains overlap
#pragma unroll
        for (int b = 0; b < kXBatch; b += 2) {
            const int u = u0 + b;
            if (u >= nunits) break;
            const bool two = u + 1 < nunits;
            __syncwarp();                                 // the previous round's pass B has read the scratch
            stage_pass_a<FMT>(v[b], u, warp, lane, xs, sw, xsum);
            if (two) stage_pass_a<FMT>(v[b + 1], u + 1, warp, lane, xs, sw + 96, xsum);
            __syncwarp();
            pass_b(u, 0);
            if (two) pass_b(u + 1, 1);
        }
    }
}

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1) quant_imma_kernel(const __grid_constant__ ImmaParams p, int stages) {
    using G = IGeom<FMT>;
    constexpr int kRS = G::kRowStride;
    constexpr int kStageBytes = G::kStageBytes;
    constexpr int kPPW = G::kPairsPerWarp;
    constexpr int kPB = IFmt<FMT>::kPairBytes;
    constexpr int kNW = IFmt<FMT>::kWordsPerRow;
    constexpr int kChunkPairs = IFmt<FMT>::kChunkPairs;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    pdl_launch_dependents();
    const int K = p.K;
    const int nchunks = K / G::kChunkCols;
    const int npairs = K / 64;
    const uint32_t base = smem_u32(smem_raw);
    uint8_t* sp = smem_raw + ((1024u - (base & 1023u)) & 1023u);
    uint8_t* stage0 = sp;
    sp += static_cast<size_t>(stages) * kStageBytes;
    uint8_t* rec = sp;                                    // [npairs][13 slots][16 B]
    sp += static_cast<size_t>(npairs) * kRecBytes;
    float* xs = reinterpret_cast<float*>(sp);             // [2 * npairs]
    sp += static_cast<size_t>(npairs) * 8;
    float* xsum = reinterpret_cast<float*>(sp);           // Q4_K: [2 * npairs] block sums, Q6_K: [4 * npairs] half sums of x
    if (FMT == FMT_Q4_K) sp += static_cast<size_t>(npairs) * 8;
    if (FMT == FMT_Q6_K) sp += static_cast<size_t>(npairs) * 16;
    float* red = reinterpret_cast<float*>(sp);            // [kRing][kCW][kRedRows]
    sp += kRing * kCW * kRedRows * 4;
    uint8_t* scratch = sp;                                // [kCW][kScratchBytes]: x staging
    sp += kCW * kScratchBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(sp);
    uint64_t* empty = full + kMaxStages;
    uint64_t* rfull = empty + kMaxStages;
    uint64_t* rempty = rfull + kRing;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = p.total_rows / kUnit;
    // units <= 2^15 (rows <= 131072), so 32-bit products suffice
    const int u_begin = static_cast<int>(static_cast<unsigned int>(units) * blockIdx.x / gridDim.x);
    const int u_end = static_cast<int>(static_cast<unsigned int>(units) * (blockIdx.x + 1) / gridDim.x);

    // The producer and epilogue warps initialise their own barriers and go
    // (bar.arrive); consumers wait for both (bar.sync) before touching them.
    // So the first weight copies leave before the rest of the CTA is set up.
    constexpr int kSetupBar = 1, kSetupThreads = kThreads;
    if (warp == kProducerWarp) {
        // Weights never depend on the previous kernel: copies start before
        // griddepcontrol.wait.  The whole warp walks the slabs; lane 0 waits
        // and arms, and the boxes of a stage go out one per lane (lane j the
        // rows 8j..8j+7, or a 4-row box for the last 4).  The first `stages`
        // fills use fresh slots (no wait).
        if (lane == 0) {
            for (int s = 0; s < stages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], kCW);
            }
            fence_mbar_init();
        }
        __syncwarp();
        named_bar_arrive(kSetupBar, kSetupThreads);
        SlabWalk walk{u_begin, u_end};
        int seg, su, nunits, s = 0, issued = 0;
        uint32_t ph = 0;
        bool alive = true;
        while (alive && walk.next(p, seg, su, nunits)) {
            const ImmaSegment& sg = p.seg[seg];
            const int r0 = su * kUnit - sg.row0;
            const int rows = nunits * kUnit;
            for (int c = 0; c < nchunks; ++c) {
                if (issued >= stages) {
                    int ok = 1;
                    if (lane == 0) ok = mbar_wait(&empty[s], ph ^ 1u) ? 1 : 0;
                    if (!__shfl_sync(0xffffffffu, ok, 0)) {
                        alive = false;
                        break;
                    }
                }
                if (lane == 0) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rows * kRS));
                __syncwarp();
                const int r = 8 * lane;
                if (r < rows)
                    tma_load_2d(smem_u32(stage0) + s * kStageBytes + r * kRS, rows - r >= 8 ? &sg.map8 : &sg.map4,
                                c * (G::kChunkBytes / 8), r0 + r, &full[s]);
                ++issued;
                if (++s == stages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        // the next launch's share of weights into L2 (all of it: this
        // keeps HBM busy across the launch boundary)
        if (lane == 0 && alive && p.prefetch) prefetch_share(p.prefetch, p.prefetch_bytes, p.prefetch_bytes);
        return;
    }

    if (warp == kEpilogueWarp) {
        // Fixed-order sum of the consumer warps' partials per slab, then bias /
        // residual and the store; lane r owns slab row r.
        if (lane == 0) {
            for (int b = 0; b < kRing; ++b) {
                mbar_init(&rfull[b], kCW);
                mbar_init(&rempty[b], 1);
            }
            fence_mbar_init();
        }
        __syncwarp();
        named_bar_arrive(kSetupBar, kSetupThreads);
        pdl_wait();
        SlabWalk walk{u_begin, u_end};
        int seg, su, nunits, sl = 0;
        float sq = 0.0f;   // deferred RMSNorm: this lane's sum of y^2
        while (walk.next(p, seg, su, nunits)) {
            const int b = sl % kRing;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&rfull[b], (sl / kRing) & 1));
            for (int r = lane; ok && r < nunits * kUnit; r += 32) {
                float acc = 0.0f;
#pragma unroll
                for (int w = 0; w < kCW; ++w) acc += red[(b * kCW + w) * kRedRows + r];
                const ImmaSegment& sg = p.seg[seg];
                const int lrow = su * kUnit + r - sg.row0;
                float out = acc;
                if (sg.bias) out += sg.bias[lrow];
                if (sg.residual) out = sg.residual[lrow] + out;
                sg.y[lrow] = out;
                if (p.norm_out) {
                    p.norm_out[lrow] = out * p.norm_w[lrow];
                    sq = fmaf(out, out, sq);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rempty[b]);
            ++sl;
        }
        if (p.norm_out) {   // the consuming launch sums the partials (fixed order) and applies the scale
            const float cta = warp_sum(sq);
            if (lane == 0) p.norm_partials[blockIdx.x] = cta;
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    named_bar(kSetupBar, kSetupThreads);
    pdl_wait();   // x comes from the previous kernel
    const int g = lane >> 2, t = lane & 3;
    const int pair_first = warp * kPPW;                   // this warp's pairs in every chunk
    if (u_begin < u_end) {
        // digits of this warp's pairs for the whole launch (read by no other warp)
        // deferred RMSNorm of x: its scale from the producer's partials (fixed order)
        float in_s = 1.0f;
        if (p.in_parts) {
            float part = 0.0f;
            for (int b = lane; b < p.in_nparts; b += 32) part += __ldcg(p.in_parts + b);
            in_s = 1.0f / sqrtf(warp_sum(part) / static_cast<float>(p.in_rows) + p.in_eps);
        }
        stage_x<FMT>(p.x, nchunks * kPPW / 2, rec, xs, scratch + warp * kScratchBytes, warp, lane, xsum, in_s);
        __syncwarp();
    }
    // Per-lane constants: offsets within a stage (row g of tile 0, pair 0 of
    // this warp); rows g + 8, tile 1 and later pairs are constant offsets.
    LaneCtx L;
    if constexpr (FMT == FMT_Q4_K) {
        // runs 2 (w % 2), 2 (w % 2) + 1 of super-block w / 2; the header
        // (d, dmin, packed scales) at the super-block's first 16 bytes
        const int sblk = (warp >> 1) * 144;
#pragma unroll
        for (int w = 0; w < 4; ++w)
            L.woff[w] = static_cast<uint32_t>(sblk + 16 + 64 * (warp & 1) + g * kRS + 16 * (t & 1) + 4 * w);
        L.v0 = static_cast<uint32_t>(sblk + g * kRS);
        L.vd = L.v0;
        L.nmask = t < 2 ? 0x0F0F0F0Fu : 0xF0F0F0F0u;
        L.oddw = static_cast<uint32_t>(warp & 1);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t sl = static_cast<uint32_t>(2 * j + (t >= 2 ? 1 : 0));   // sub-block mod 4
            L.ksel[j] = sl | (sl + 4u) << 4;
        }
        L.xsum_off = static_cast<uint32_t>(npairs) * 8u;
        L.kmin = (t & 1) ? 0.0f : 1.0f;
    } else if constexpr (FMT == FMT_Q6_K) {
        // super-block w / 2 (byte B of the chunk row), half h = w % 2; lane
        // values i0..i0+7 of each block (i0 = 16 (t / 2) + 8 (t % 2))
        const int sbB = (warp >> 1) * 210, h = warp & 1, half = t >> 1;
        const int i0 = 16 * half + 8 * (t & 1), off = sbB & 3;   // off: 0 or 2
        const int rowg = g * kRS;
        L.qoff[0] = static_cast<uint32_t>(rowg + sbB + 64 * h + i0 - off);
        L.qoff[1] = static_cast<uint32_t>(rowg + sbB + 64 * h + 32 + i0 - off);
        L.qoff[2] = static_cast<uint32_t>(rowg + sbB + 128 + 32 * h + i0 - off);
        const int s0 = sbB + 192 + 8 * h + half, sa = s0 & ~3;   // scales[8h + 2k + half], k = 2J + m
        L.soff = static_cast<uint32_t>(rowg + sa);
        L.sw = 0u;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int pb = s0 - sa + 2 * e;
            const uint32_t idx = static_cast<uint32_t>(pb < 8 ? pb : pb - 4);
            if (pb >= 8) L.sw |= 1u << e;
            L.ssel[e] = idx | (8u | idx) << 4 | (8u | idx) << 8 | (8u | idx) << 12;
        }
        const int dp = sbB + 208;
        L.doff = static_cast<uint32_t>(rowg + (dp & ~3));
        L.dsh = (dp & 3) ? 16u : 0u;
        L.oddw = off != 0 ? 1u : 0u;
        L.kmin = (t & 1) ? 0.0f : 1.0f;
        L.nmask = 0u;
        L.ksel[0] = L.ksel[1] = 0u;
        L.xsum_off = 0u;
    } else {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const int sw = w < kNW ? src_word(FMT, t, w) : 0;
            L.woff[w] =
                static_cast<uint32_t>(pair_first * kPB + g * kRS + 4 * (sw >= 0 ? sw : (FMT == FMT_Q4_0 ? 4 : 8)));
        }
        L.v0 = static_cast<uint32_t>(pair_first * kPB + g * kRS);
        L.vd = L.v0 + (FMT == FMT_Q4_0 ? 16u : 32u);
        L.nmask = 0u;
        L.oddw = 0u;
        L.ksel[0] = L.ksel[1] = 0u;
        L.xsum_off = 0u;
        L.kmin = 0.0f;
    }
    L.sel_fix = t == 1 ? 0x1076u : 0x3210u;
    L.sel_d = t < 2 ? 0x3210u : 0x7676u;
    const bool bact = t < 2 ? g < 3 : (g >= 4 && g < 7);
    const int slot = bact ? (t < 2 ? 2 * g + t : 6 + 2 * (g - 4) + (t - 2)) : kZeroSlot;
    L.brec = smem_u32(rec) + slot * 16;
    L.xsl = smem_u32(xs) + (FMT == FMT_Q6_K ? 0u : 4u * (t >> 1));   // Q6_K: MMA m is block m for every lane
    L.xs16l = smem_u32(xsum) + 4u * (t >> 1);
    L.kd0 = mk2((t & 1) ? 1.0f : 65536.0f, (t & 1) ? 1.0f : 65536.0f);
    L.kd1 = mk2((t & 1) ? 0.0f : 256.0f, (t & 1) ? 0.0f : 256.0f);
    if (FMT == FMT_Q4_K && t >= 2) {   // high nibbles enter as 16 c
        L.kd0 = mul2(L.kd0, mk2(0.0625f, 0.0625f));
        L.kd1 = mul2(L.kd1, mk2(0.0625f, 0.0625f));
    }
    const uint32_t stage_s = smem_u32(stage0);

    SlabWalk walk{u_begin, u_end};
    int seg, su, nunits, s = 0, sl = 0;
    uint32_t ph = 0;
    while (walk.next(p, seg, su, nunits)) {
        const int ntiles = (nunits * kUnit + 15) / 16;    // 1, 2 or 3 (warp-uniform)
        f2 y0 = mk2(0.0f, 0.0f), y1 = mk2(0.0f, 0.0f), y2 = mk2(0.0f, 0.0f);   // rows (g, g+8), (g+16, g+24), (g+32, -)
        for (int c = 0; c < nchunks; ++c) {
            const int P0 = c * kChunkPairs + pair_first;
            // warp-uniform: the MMAs below need all 32 lanes
            if (__all_sync(0xffffffffu, mbar_wait(&full[s], ph))) {
                const uint32_t sb = stage_s + s * kStageBytes;
                const uint32_t st[4] = {sb + L.woff[0], sb + L.woff[1], sb + L.woff[2], sb + L.woff[3]};
                const uint32_t pb = L.brec + P0 * kRecBytes, px = L.xsl + 8u * P0;
                if constexpr (FMT == FMT_Q4_K) {
                    if (ntiles == 2)
                        stage_pairs_k<2>(L, st[0], sb + L.v0, pb, px, y0, y1, y2);
                    else if (ntiles == 1)
                        stage_pairs_k<1>(L, st[0], sb + L.v0, pb, px, y0, y1, y2);
                    else
                        stage_pairs_k<3>(L, st[0], sb + L.v0, pb, px, y0, y1, y2);
                } else if constexpr (FMT == FMT_Q6_K) {
                    const uint32_t px16 = L.xs16l + 16u * P0;
                    if (ntiles == 2)
                        stage_pairs_q6<2>(L, sb, pb, px, px16, y0, y1, y2);
                    else if (ntiles == 1)
                        stage_pairs_q6<1>(L, sb, pb, px, px16, y0, y1, y2);
                    else
                        stage_pairs_q6<3>(L, sb, pb, px, px16, y0, y1, y2);
                } else {
                    if (ntiles == 2)
                        stage_pairs<FMT, 2>(L, st, sb + L.v0, sb + L.vd, pb, px, y0, y1, y2);
                    else if (ntiles == 1)
                        stage_pairs<FMT, 1>(L, st, sb + L.v0, sb + L.vd, pb, px, y0, y1, y2);
                    else
                        stage_pairs<FMT, 3>(L, st, sb + L.v0, sb + L.vd, pb, px, y0, y1, y2);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == stages) {
                s = 0;
                ph ^= 1u;
            }
        }
        float r[5] = {lo(y0), hi(y0), lo(y1), hi(y1), lo(y2)};
#pragma unroll
        for (int i = 0; i < 5; ++i) {
            r[i] += __shfl_xor_sync(0xffffffffu, r[i], 1);
            r[i] += __shfl_xor_sync(0xffffffffu, r[i], 2);
        }
        const int b = sl % kRing;
        mbar_wait(&rempty[b], ((sl / kRing) & 1) ^ 1u);
        if (t == 0) {
            float* rr = red + (b * kCW + warp) * kRedRows;
            rr[g] = r[0];
            rr[g + 8] = r[1];
            rr[g + 16] = r[2];
            rr[g + 24] = r[3];
            if (g < 4) rr[g + 32] = r[4];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rfull[b]);
        ++sl;
    }
}

template <int FMT>
bool encode_maps(ImmaSegment& ms, const void* w, int K, int rows) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    const size_t row_bytes = FMT == FMT_Q6_K ? static_cast<size_t>(K) / 256 * 210
                                             : static_cast<size_t>(K) / 32 * (FMT == FMT_Q8_0 ? 34 : 18);   // Q4_K: K / 256 * 144
    const cuuint64_t dims[2] = {row_bytes / 8, static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t es[2] = {1, 1};
    for (int v = 0; v < 2; ++v) {
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(IGeom<FMT>::kBoxElems), v == 0 ? 8u : 4u};
        if (fn(v == 0 ? &ms.map8 : &ms.map4, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides,
               box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

int stage_bytes_of(int fmt) {
    return fmt == FMT_Q4_0   ? IGeom<FMT_Q4_0>::kStageBytes
           : fmt == FMT_Q4_K ? IGeom<FMT_Q4_K>::kStageBytes
           : fmt == FMT_Q6_K ? IGeom<FMT_Q6_K>::kStageBytes
                             : IGeom<FMT_Q8_0>::kStageBytes;
}

size_t fixed_smem(int fmt, int K) {
    const size_t npairs = static_cast<size_t>(K / 64);
    return 1024 + npairs * (kRecBytes + (fmt == FMT_Q4_K ? 16 : fmt == FMT_Q6_K ? 24 : 8)) + kRing * kCW * kRedRows * 4 +
           kCW * kScratchBytes +
           (2 * kMaxStages + 2 * kRing) * 8;
}

// Stages (at most kMaxStages) that fit beside the fixed part in 227 KB.
void plan_smem(int fmt, int K, int* stages, size_t* smem) {
    const size_t fixed = fixed_smem(fmt, K);
    const int sb = stage_bytes_of(fmt);
    *stages = static_cast<int>(std::min<size_t>(kMaxStages, kSmemMax > fixed ? (kSmemMax - fixed) / sb : 0));
    *smem = fixed + static_cast<size_t>(*stages) * sb;
}

}  // namespace

bool matvec_imma_supported(int fmt, int K) {
    if ((fmt != FMT_Q4_0 && fmt != FMT_Q8_0 && fmt != FMT_Q4_K && fmt != FMT_Q6_K) || K <= 0 || K % 2048 != 0)
        return false;
    int stages = 0;
    size_t smem = 0;
    plan_smem(fmt, K, &stages, &smem);
    if (stages < 2) return false;
    return tensor_map_encoder() != nullptr;
}

cudaError_t launch_matvec_imma(int fmt, const MatvecParams& mp, cudaStream_t stream, bool pdl) {
    if (!matvec_imma_supported(fmt, mp.K)) return cudaErrorNotSupported;
    if (mp.epilogue != EPI_STORE || mp.tpl.tp > 1) return cudaErrorNotSupported;
    // RMSNorm only deferred (no last-CTA pass), on a single segment
    if (mp.norm_out && (!mp.norm_defer || mp.nseg != 1 || !mp.norm_w || !mp.norm_partials))
        return cudaErrorNotSupported;
    if (mp.norm_defer && !mp.norm_out) return cudaErrorNotSupported;
    if (mp.in_parts && (mp.in_nparts <= 0 || mp.in_rows <= 0)) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(mp.x) & 15) != 0) return cudaErrorNotSupported;
    for (int s = 0; s < mp.nseg; ++s)
        if (mp.seg[s].rows % kUnit != 0 || (reinterpret_cast<uintptr_t>(mp.seg[s].w) & 15) != 0)
            return cudaErrorNotSupported;
    ImmaParams p;
    memset(&p, 0, sizeof p);
    p.nseg = mp.nseg;
    p.K = mp.K;
    p.total_rows = mp.total_rows;
    p.x = mp.x;
    p.prefetch = static_cast<const uint8_t*>(mp.prefetch);
    p.prefetch_bytes = mp.prefetch_bytes;
    p.norm_out = mp.norm_out;
    p.norm_w = mp.norm_w;
    p.norm_partials = mp.norm_partials;
    p.in_parts = mp.in_parts;
    p.in_nparts = mp.in_nparts;
    p.in_rows = mp.in_rows;
    p.in_eps = mp.in_eps;
    int row0 = 0;
    for (int s = 0; s < mp.nseg; ++s) {
        ImmaSegment& ms = p.seg[s];
        const bool ok = fmt == FMT_Q4_0   ? encode_maps<FMT_Q4_0>(ms, mp.seg[s].w, mp.K, mp.seg[s].rows)
                        : fmt == FMT_Q4_K ? encode_maps<FMT_Q4_K>(ms, mp.seg[s].w, mp.K, mp.seg[s].rows)
                        : fmt == FMT_Q6_K ? encode_maps<FMT_Q6_K>(ms, mp.seg[s].w, mp.K, mp.seg[s].rows)
                                          : encode_maps<FMT_Q8_0>(ms, mp.seg[s].w, mp.K, mp.seg[s].rows);
        if (!ok) return cudaErrorInvalidValue;
        ms.bias = mp.seg[s].bias;
        ms.residual = mp.seg[s].residual;
        ms.y = mp.seg[s].y;
        ms.rows = mp.seg[s].rows;
        ms.row0 = row0;
        row0 += mp.seg[s].rows;
    }
    int stages = 0;
    size_t smem = 0;
    plan_smem(fmt, mp.K, &stages, &smem);
    auto kern = fmt == FMT_Q4_0   ? quant_imma_kernel<FMT_Q4_0>
                : fmt == FMT_Q4_K ? quant_imma_kernel<FMT_Q4_K>
                : fmt == FMT_Q6_K ? quant_imma_kernel<FMT_Q6_K>
                                  : quant_imma_kernel<FMT_Q8_0>;
    static bool configured[4][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    bool& done = configured[fmt == FMT_Q4_0 ? 0 : fmt == FMT_Q4_K ? 2 : fmt == FMT_Q6_K ? 3 : 1][dev & 63];
    if (!done) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        done = true;
    }
    const int units = mp.total_rows / kUnit;
    const int grid = std::max(1, std::min(sm_count_for_current_device(), units));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p, stages);
}

}  // namespace alj
