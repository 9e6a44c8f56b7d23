/*
 * aljabr_oracle.c -- TEST INFRASTRUCTURE ONLY (see aljabr_oracle.h).
 *
 * Compiled with -ffp-contract=off so that every `a * b + c` rounds twice,
 * as Java float arithmetic does; fused multiply-adds appear only where the
 * reference itself calls Math.fma or FloatVector.fma.
 *
 * Where the reference uses the Java Vector API, the lane width follows the
 * species it names: GGUFVectorOps uses SPECIES_PREFERRED (machine
 * dependent; restated here as 8 lanes, the AVX2 width) and the Q8 raw dot
 * uses SPECIES_256 (8 float lanes).  reduceLanes(ADD) has no specified
 * order; it is restated as a left-to-right lane sum.
 */
#include "aljabr_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define VLANES 8

static const float NF4_TABLE[16] = {
    /* engine/safetensor/.../DequantizationKernel.java:23-28 */
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

static inline float f32_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t bits_of(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
static inline uint16_t le16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------------------------ */
/* RT/GgufQuantTables.java:143-165 (f16ToF32Slow; the 64K table is built from it). */
float orc_f16_to_f32(uint16_t half) {
    int sign = (half >> 15) & 1;
    int exponent = (half >> 10) & 0x1F;
    int mantissa = half & 0x3FF;
    if (exponent == 0) {
        if (mantissa == 0) return sign ? -0.0f : 0.0f;
        float value = ldexpf((float)mantissa / 1024.0f, -14);   /* Math.scalb, exact */
        return sign ? -value : value;
    }
    if (exponent == 31) {
        if (mantissa == 0) return sign ? -INFINITY : INFINITY;
        return f32_from_bits(0x7FC00000u);                       /* Float.NaN */
    }
    return f32_from_bits(((uint32_t)sign << 31) | ((uint32_t)(exponent + 112) << 23) | ((uint32_t)mantissa << 13));
}

/* GW:360-387.  Float.floatToIntBits canonicalises NaN first. */
uint16_t orc_f32_to_f16_bits(float value) {
    uint32_t bits = bits_of(value);
    if (value != value) bits = 0x7FC00000u;
    int sign = (int)((bits >> 16) & 0x8000);
    int exponent = (int)((bits >> 23) & 0xFF) - 127 + 15;
    int mantissa = (int)(bits & 0x7FFFFF);
    if (exponent >= 31) return (uint16_t)(sign | 0x7C00 | (mantissa == 0 ? 0 : 1));
    if (exponent <= 0) {
        if (exponent < -10) return (uint16_t)sign;
        mantissa |= 0x800000;
        int shift = 14 - exponent;
        int half_mantissa = mantissa >> shift;
        if (((mantissa >> (shift - 1)) & 1) != 0) half_mantissa++;
        return (uint16_t)(sign | half_mantissa);
    }
    int half = sign | (exponent << 10) | (mantissa >> 13);
    if ((mantissa & 0x1000) != 0) half++;
    return (uint16_t)half;
}

/* java.lang.Math.round(float): nearest int, ties toward +inf, NaN -> 0,
 * saturating.  floor(a + 0.5) in double is exact for every float. */
int orc_java_round(float value) {
    if (value != value) return 0;
    double r = floor((double)value + 0.5);
    if (r >= 2147483647.0) return 2147483647;
    if (r <= -2147483648.0) return (int)-2147483648LL;
    return (int)r;
}

uint16_t orc_f32_to_bf16_rne(float value) {
    uint32_t b = bits_of(value);
    if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((b >> 16) | 0x40);   /* quiet NaN */
    uint32_t lsb = (b >> 16) & 1u;
    b += 0x7FFFu + lsb;
    return (uint16_t)(b >> 16);
}

static inline float bf16_to_f32(uint16_t h) { return f32_from_bits((uint32_t)h << 16); }

/* ------------------------------------------------------------------------ */
static float java_max_abs(const float* v, int n) {            /* GW:196-202 */
    float m = 0.0f;
    for (int i = 0; i < n; i++) {
        float a = fabsf(v[i]);
        if (a != a) { m = a; continue; }                       /* Math.max propagates NaN */
        if (m != m) continue;
        if (a > m) m = a;
    }
    return m;
}
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

void orc_encode_q8_0(const float* values, int64_t n, uint8_t* out) {   /* GW:163-177 */
    for (int64_t block = 0; block < n; block += 32) {
        float scale = java_max_abs(values + block, 32) / 127.0f;
        uint16_t h = orc_f32_to_f16_bits(scale);
        out[0] = (uint8_t)(h & 0xFF); out[1] = (uint8_t)(h >> 8);
        for (int i = 0; i < 32; i++) {
            int q = scale == 0.0f ? 0 : orc_java_round(values[block + i] / scale);
            out[2 + i] = (uint8_t)(clampi(q, -127, 127) & 0xFF);
        }
        out += 34;
    }
}

static int quantize4(float value, float scale) {              /* GW:204-209 */
    if (scale == 0.0f) return 0;
    return clampi(orc_java_round(value / scale), -8, 7);
}

void orc_encode_q4_0(const float* values, int64_t n, uint8_t* out) {   /* GW:179-194 */
    for (int64_t block = 0; block < n; block += 32) {
        float scale = java_max_abs(values + block, 32) / 7.0f;
        uint16_t h = orc_f32_to_f16_bits(scale);
        out[0] = (uint8_t)(h & 0xFF); out[1] = (uint8_t)(h >> 8);
        for (int i = 0; i < 16; i++) {
            int lo = quantize4(values[block + i], scale) + 8;
            int hi = quantize4(values[block + 16 + i], scale) + 8;
            out[2 + i] = (uint8_t)((hi << 4) | lo);
        }
        out += 18;
    }
}

void orc_quantize_nf4(const float* values, int64_t n, int group_size, uint8_t* codes, float* absmax) {
    int64_t groups = (n + group_size - 1) / group_size;
    for (int64_t g = 0; g < groups; g++) {
        int64_t start = g * group_size;
        int len = (int)((start + group_size <= n) ? group_size : n - start);
        absmax[g] = java_max_abs(values + start, len);
    }
    for (int64_t i = 0; i < n; i++) {
        float s = absmax[i / group_size];
        int best = 7;
        if (s != 0.0f) {
            float v = values[i] / s;
            float bestd = INFINITY;
            for (int c = 0; c < 16; c++) {
                float d = fabsf(NF4_TABLE[c] - v);
                if (d < bestd) { bestd = d; best = c; }
            }
        }
        if ((i & 1) == 0) codes[i >> 1] = (uint8_t)(best << 4);
        else codes[i >> 1] |= (uint8_t)best;
    }
}

/* ------------------------------------------------------------------------ */
/* DK:84-102.  The odd element reuses the even element's group index. */
void orc_dequantize_nf4(const uint8_t* src, float* dst, const float* scales, int64_t numel, int group_size) {
    int64_t num_bytes = (numel + 1) / 2;
    for (int64_t i = 0; i < num_bytes; i++) {
        int b = src[i];
        int v1 = (b >> 4) & 0x0F;
        int v2 = b & 0x0F;
        float scale = scales[(i * 2) / group_size];
        dst[i * 2] = NF4_TABLE[v1] * scale;
        if (i * 2 + 1 < numel) dst[i * 2 + 1] = NF4_TABLE[v2] * scale;
    }
}

/* RT/GgufBlockDequantizer.java:33-37 -> dequantizeQ4Block :366-415 with
 * zeroPoint 8 and bias +0.0f (the bias add turns -0.0 into +0.0). */
void orc_dequantize_q4_0(const uint8_t* blocks, float* dst, int64_t numel) {
    for (int64_t b = 0; b < numel / 32; b++) {
        const uint8_t* blk = blocks + b * 18;
        float d = orc_f16_to_f32(le16(blk));
        float* o = dst + b * 32;
        for (int j = 0; j < 16; j++) {
            int quant = blk[2 + j];
            o[j] = (float)((quant & 0x0F) - 8) * d + 0.0f;
            o[16 + j] = (float)((quant >> 4) - 8) * d + 0.0f;
        }
    }
}

/* RT/GgufRowDequantizer.java:142-151 -> GgufBlockDequantizer.java:231-265. */
void orc_dequantize_q8_0(const uint8_t* blocks, float* dst, int64_t numel) {
    for (int64_t b = 0; b < numel / 32; b++) {
        const uint8_t* blk = blocks + b * 34;
        float d = orc_f16_to_f32(le16(blk));
        for (int j = 0; j < 32; j++) dst[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
    }
}

/* ------------------------------------------------------------------------ */
/* RT/GgufQ32RawDot.java:454-462 (dotQ4_0PackedNibbleByte). */
static inline float q4_nibble_byte(int quant, const float* v, int index) {
    return (float)((quant & 0x0F) - 8) * v[index] + (float)((quant >> 4) - 8) * v[16 + index];
}

/* RT/GgufQ32RawDot.java:428-452: byte i of the 16 code bytes feeds lane
 * i % 4; each lane sums its four bytes left to right. */
static float q4_0_unscaled_block(const uint8_t* codes, const float* v) {
    float s[4];
    for (int lane = 0; lane < 4; lane++) {
        s[lane] = q4_nibble_byte(codes[lane], v, lane) + q4_nibble_byte(codes[4 + lane], v, 4 + lane)
                + q4_nibble_byte(codes[8 + lane], v, 8 + lane) + q4_nibble_byte(codes[12 + lane], v, 12 + lane);
    }
    return s[0] + s[1] + s[2] + s[3];
}

static inline float q4_0_block(const uint8_t* blk, const float* v) {   /* :342-348 */
    float d = orc_f16_to_f32(le16(blk));
    return d * q4_0_unscaled_block(blk + 2, v);
}

float orc_dot_row_q4_0(const uint8_t* row, int columns, const float* x) {   /* :34-67 */
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int blocks = columns / 32, block = 0, unrolled_limit = blocks - 4;
    for (; block <= unrolled_limit; block += 4) {
        s0 += q4_0_block(row + (size_t)block * 18, x + block * 32);
        s1 += q4_0_block(row + (size_t)(block + 1) * 18, x + (block + 1) * 32);
        s2 += q4_0_block(row + (size_t)(block + 2) * 18, x + (block + 2) * 32);
        s3 += q4_0_block(row + (size_t)(block + 3) * 18, x + (block + 3) * 32);
    }
    float sum = s0 + s1 + s2 + s3;
    for (; block < blocks; block++) sum += q4_0_block(row + (size_t)block * 18, x + block * 32);
    return sum;
}

/* RT/GgufQ8RawDot.java:784-830: lane l sums bytes l, l+4, l+8, ... in pairs. */
static float q8_unscaled_block_scalar(const uint8_t* q, const float* v) {
    float s[4];
    for (int lane = 0; lane < 4; lane++) {
        float acc = (float)(int8_t)q[lane] * v[lane] + (float)(int8_t)q[lane + 4] * v[lane + 4];
        acc += (float)(int8_t)q[lane + 8] * v[lane + 8] + (float)(int8_t)q[lane + 12] * v[lane + 12];
        acc += (float)(int8_t)q[lane + 16] * v[lane + 16] + (float)(int8_t)q[lane + 20] * v[lane + 20];
        acc += (float)(int8_t)q[lane + 24] * v[lane + 24] + (float)(int8_t)q[lane + 28] * v[lane + 28];
        s[lane] = acc;
    }
    return s[0] + s[1] + s[2] + s[3];
}

float orc_dot_row_q8_0_scalar(const uint8_t* row, int columns, const float* x) {   /* :138-185 */
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int blocks = columns / 32, block = 0, unrolled_limit = blocks - 4;
    for (; block <= unrolled_limit; block += 4) {
        for (int u = 0; u < 4; u++) {
            const uint8_t* blk = row + (size_t)(block + u) * 34;
            float t = orc_f16_to_f32(le16(blk)) * q8_unscaled_block_scalar(blk + 2, x + (block + u) * 32);
            if (u == 0) s0 += t; else if (u == 1) s1 += t; else if (u == 2) s2 += t; else s3 += t;
        }
    }
    float sum = s0 + s1 + s2 + s3;
    for (; block < blocks; block++) {
        const uint8_t* blk = row + (size_t)block * 34;
        float d = orc_f16_to_f32(le16(blk));
        sum += d * q8_unscaled_block_scalar(blk + 2, x + block * 32);
    }
    return sum;
}

/* RT/GgufQ8RawDot.java:755-782: one block into an 8-lane accumulator. */
static void q8_block_vector(const uint8_t* q, const float* v, float scale, float* acc) {
    for (int l = 0; l < VLANES; l++) {
        float b = (float)(int8_t)q[l] * v[l];
        b = fmaf((float)(int8_t)q[8 + l], v[8 + l], b);
        b = fmaf((float)(int8_t)q[16 + l], v[16 + l], b);
        b = fmaf((float)(int8_t)q[24 + l], v[24 + l], b);
        acc[l] = fmaf(b, scale, acc[l]);
    }
}

float orc_dot_row_q8_0_vector(const uint8_t* row, int columns, const float* x) {   /* :63-121 */
    float a[4][VLANES];
    memset(a, 0, sizeof a);
    int blocks = columns / 32, block = 0, unrolled_limit = blocks - 4;
    for (; block <= unrolled_limit; block += 4)
        for (int u = 0; u < 4; u++) {
            const uint8_t* blk = row + (size_t)(block + u) * 34;
            q8_block_vector(blk + 2, x + (block + u) * 32, orc_f16_to_f32(le16(blk)), a[u]);
        }
    float acc[VLANES];
    for (int l = 0; l < VLANES; l++) acc[l] = a[0][l] + a[1][l] + a[2][l] + a[3][l];
    for (; block < blocks; block++) {
        const uint8_t* blk = row + (size_t)block * 34;
        q8_block_vector(blk + 2, x + block * 32, orc_f16_to_f32(le16(blk)), acc);
    }
    float r = 0.0f;
    for (int l = 0; l < VLANES; l++) r += acc[l];
    return r;
}

/* ------------------------------------------------------------------------ */
/* K-quants: 256-value super-blocks.
 * Q4_K (144 B): fp16 d, fp16 dmin, 12 bytes of packed 6-bit (scale, min)
 * pairs for 8 sub-blocks of 32, 128 bytes of nibbles; the 64 values of
 * chunk j take the low nibbles (sub-block 2j) then the high nibbles
 * (sub-block 2j+1) of bytes [32j, 32j+32).  value = d*scale*q - dmin*min.
 * Q6_K (210 B): ql[128] low nibbles, qh[64] two-bit high parts, int8
 * scales[16] (one per 16 values), fp16 d at byte 208.  In each 128-value
 * half h, value 32k + i (k < 4, i < 32) is ql[64h + 32(k&1) + i] nibble
 * (k >> 1) with bits 2k..2k+1 of qh[32h + i] on top, minus 32, times
 * d * scales[8h + 2k + i/16]. */

/* RT/GgufKQuantLayout.java:37-50 (scaleMinK4PackedCode) and :60-66 (scaleK4Packed). */
static void q4k_scale_min(const uint8_t* sc, int index, int* scale, int* min) {
    if (index < 4) {
        *scale = sc[index] & 63;
        *min = sc[index + 4] & 63;
    } else {
        *scale = (sc[index + 4] & 0x0F) | ((sc[index - 4] >> 6) << 4);
        *min = (sc[index + 4] >> 4) | ((sc[index] >> 6) << 4);
    }
}

/* RT/GgufQ4RawDot.java:38-141 (dotRowQ4K): per 64-value chunk two 8-wide
 * left-to-right product sums per step, the vector sums only where a min is
 * non-zero, then sum += d1*dot1 + d2*dot2 and the min corrections. */
float orc_dot_row_q4_k(const uint8_t* row, int columns, const float* x) {
    float sum = 0.0f;
    for (int b = 0; b < columns / 256; b++) {
        const uint8_t* blk = row + (int64_t)b * 144;
        const float d = orc_f16_to_f32(le16(blk));
        const float dmin = orc_f16_to_f32(le16(blk + 2));
        const int block_mins = dmin != 0.0f;
        const uint8_t* qs = blk + 16;
        const float* v = x + (int64_t)b * 256;
        for (int j = 0; j < 4; j++) {
            int s1, m1, s2, m2;
            q4k_scale_min(blk + 4, 2 * j, &s1, &m1);
            q4k_scale_min(blk + 4, 2 * j + 1, &s2, &m2);
            const float d1 = d * (float)s1, d2 = d * (float)s2;
            const int min1 = block_mins ? m1 : 0, min2 = block_mins ? m2 : 0;
            const int has1 = block_mins && min1 != 0, has2 = block_mins && min2 != 0;
            float vs1 = 0.0f, vs2 = 0.0f, dot1 = 0.0f, dot2 = 0.0f;
            for (int i = 0; i < 32; i += 8) {
                float t1 = (float)(qs[i] & 0x0F) * v[i];
                float t2 = (float)((qs[i] >> 4) & 0x0F) * v[32 + i];
                for (int k = 1; k < 8; k++) {
                    t1 = t1 + (float)(qs[i + k] & 0x0F) * v[i + k];
                    t2 = t2 + (float)((qs[i + k] >> 4) & 0x0F) * v[32 + i + k];
                }
                dot1 += t1;
                dot2 += t2;
                if (has1) {
                    float u = v[i];
                    for (int k = 1; k < 8; k++) u = u + v[i + k];
                    vs1 += u;
                }
                if (has2) {
                    float u = v[32 + i];
                    for (int k = 1; k < 8; k++) u = u + v[32 + i + k];
                    vs2 += u;
                }
            }
            sum += d1 * dot1 + d2 * dot2;
            if (has1) sum -= dmin * (float)min1 * vs1;
            if (has2) sum -= dmin * (float)min2 * vs2;
            qs += 32;
            v += 64;
        }
    }
    return sum;
}

/* RT/GgufQ6RawDot.java:403-513 (dotRowQ6KHalf): 16 values of each of the
 * four 32-value quarters of a half, 8-wide left-to-right product sums. */
static float q6k_half(const uint8_t* ql, const uint8_t* qh, const float* v, int off,
                      float s1, float s2, float s3, float s4) {
    float dot1 = 0.0f, dot2 = 0.0f, dot3 = 0.0f, dot4 = 0.0f;
    for (int i = off; i < off + 16; i += 8) {
        float t[4] = {0, 0, 0, 0};
        for (int k = 0; k < 8; k++) {
            const int a = ql[i + k], c = ql[32 + i + k], h = qh[i + k];
            const float p1 = (float)(((a & 0x0F) | ((h & 3) << 4)) - 32) * v[i + k];
            const float p2 = (float)(((c & 0x0F) | (((h >> 2) & 3) << 4)) - 32) * v[32 + i + k];
            const float p3 = (float)(((a >> 4) | (((h >> 4) & 3) << 4)) - 32) * v[64 + i + k];
            const float p4 = (float)(((c >> 4) | (((h >> 6) & 3) << 4)) - 32) * v[96 + i + k];
            if (k == 0) { t[0] = p1; t[1] = p2; t[2] = p3; t[3] = p4; }
            else { t[0] = t[0] + p1; t[1] = t[1] + p2; t[2] = t[2] + p3; t[3] = t[3] + p4; }
        }
        dot1 += t[0];
        dot2 += t[1];
        dot3 += t[2];
        dot4 += t[3];
    }
    return s1 * dot1 + s2 * dot2 + s3 * dot3 + s4 * dot4;
}

/* RT/GgufQ6RawDot.java:77-133 (dotRowQ6KBlock). */
static float q6k_block(const uint8_t* blk, const float* v) {
    const float d = orc_f16_to_f32(le16(blk + 208));
    const int8_t* sc = (const int8_t*)(blk + 192);
    const float s0 = q6k_half(blk, blk + 128, v, 0, d * sc[0], d * sc[2], d * sc[4], d * sc[6]);
    const float s1 = q6k_half(blk, blk + 128, v, 16, d * sc[1], d * sc[3], d * sc[5], d * sc[7]);
    const float s2 = q6k_half(blk + 64, blk + 160, v + 128, 0, d * sc[8], d * sc[10], d * sc[12], d * sc[14]);
    const float s3 = q6k_half(blk + 64, blk + 160, v + 128, 16, d * sc[9], d * sc[11], d * sc[13], d * sc[15]);
    return s0 + s1 + s2 + s3;
}

/* RT/GgufQ6RawDot.java:33-75 (dotRowQ6K): four running block sums, then the tail. */
float orc_dot_row_q6_k(const uint8_t* row, int columns, const float* x) {
    const int blocks = columns / 256;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    int b = 0;
    for (; b <= blocks - 4; b += 4) {
        a0 += q6k_block(row + (int64_t)b * 210, x + (int64_t)b * 256);
        a1 += q6k_block(row + (int64_t)(b + 1) * 210, x + (int64_t)(b + 1) * 256);
        a2 += q6k_block(row + (int64_t)(b + 2) * 210, x + (int64_t)(b + 2) * 256);
        a3 += q6k_block(row + (int64_t)(b + 3) * 210, x + (int64_t)(b + 3) * 256);
    }
    float sum = a0 + a1 + a2 + a3;
    for (; b < blocks; b++) sum += q6k_block(row + (int64_t)b * 210, x + (int64_t)b * 256);
    return sum;
}

/* Values of one K-quant row (element formulas above), for fp64 sums and tests. */
void orc_dequantize_k_row(int type, const uint8_t* row, int columns, double* out) {
    for (int b = 0; b < columns / 256; b++) {
        double* o = out + (int64_t)b * 256;
        if (type == ORC_Q4_K) {
            const uint8_t* blk = row + (int64_t)b * 144;
            const double d = orc_f16_to_f32(le16(blk)), dmin = orc_f16_to_f32(le16(blk + 2));
            for (int e = 0; e < 256; e++) {
                const int j = e / 64, t = e % 64, sb = 2 * j + (t >= 32);
                const int byte = blk[16 + 32 * j + (t & 31)];
                const int q = t < 32 ? (byte & 15) : (byte >> 4);
                int sc, mn;
                q4k_scale_min(blk + 4, sb, &sc, &mn);
                o[e] = d * sc * q - dmin * mn;
            }
        } else {
            const uint8_t* blk = row + (int64_t)b * 210;
            const double d = orc_f16_to_f32(le16(blk + 208));
            for (int e = 0; e < 256; e++) {
                const int h = e / 128, w = e % 128, k = w / 32, i = w % 32;
                const int lo = blk[64 * h + 32 * (k & 1) + i];
                const int hb = blk[128 + 32 * h + i];
                const int q = (((k >> 1) ? (lo >> 4) : (lo & 15)) | (((hb >> (2 * k)) & 3) << 4)) - 32;
                o[e] = d * (int8_t)blk[192 + 8 * h + 2 * k + i / 16] * q;
            }
        }
    }
}

/* ---- Q4_0 prepared path: the reference's default for >= 32 rows --------
 * RT/GgufPreparedCachePolicy.java:66-75 (cache_min_rows 32) selects the
 * prepared matrix built by RT/GgufQ32Build.java:78-91 (fillQ4_0Blocks: fp32
 * block scale f16ToF32(d); codes unpacked by RT/GgufQuantUnpacker.java:
 * 365-367,414-433,445-448 to int8 (q & 15) - 8 at index i and (q >> 4) - 8
 * at index 16 + i), then dotted by RT/GgufQ32Dot.java:627-670
 * (dotRowQ32PreparedNoBiasScalar: four interleaved Math.fma accumulators
 * over blocks, sum0 + sum1 + sum2 + sum3, fma tail) with the per-block dot
 * RT/GgufDot.java:1046-1058 (dotSignedByte32Scalar: four lane partial sums
 * of int8 * float, lane sum left to right). */
static float q4_0_prepared_block_dot(const uint8_t* blk, const float* v) {
    int8_t q[32];
    for (int i = 0; i < 16; i++) {
        const int b = blk[2 + i];
        q[i] = (int8_t)((b & 0x0F) - 8);
        q[16 + i] = (int8_t)((b >> 4) - 8);
    }
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    for (int i = 0; i < 32; i += 4) {
        s0 += (float)q[i] * v[i];
        s1 += (float)q[i + 1] * v[i + 1];
        s2 += (float)q[i + 2] * v[i + 2];
        s3 += (float)q[i + 3] * v[i + 3];
    }
    return s0 + s1 + s2 + s3;
}
float orc_dot_row_q4_0_prepared(const uint8_t* row, int columns, const float* x) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int blocks = columns / 32, block = 0, unrolled_limit = blocks - 4;
    for (; block <= unrolled_limit; block += 4) {
        const uint8_t* b = row + (size_t)block * 18;
        s0 = fmaf(orc_f16_to_f32(le16(b)), q4_0_prepared_block_dot(b, x + block * 32), s0);
        s1 = fmaf(orc_f16_to_f32(le16(b + 18)), q4_0_prepared_block_dot(b + 18, x + (block + 1) * 32), s1);
        s2 = fmaf(orc_f16_to_f32(le16(b + 36)), q4_0_prepared_block_dot(b + 36, x + (block + 2) * 32), s2);
        s3 = fmaf(orc_f16_to_f32(le16(b + 54)), q4_0_prepared_block_dot(b + 54, x + (block + 3) * 32), s3);
    }
    float sum = s0 + s1 + s2 + s3;
    for (; block < blocks; block++) {
        const uint8_t* b = row + (size_t)block * 18;
        sum = fmaf(orc_f16_to_f32(le16(b)), q4_0_prepared_block_dot(b, x + block * 32), sum);
    }
    return sum;
}

/* ---- the FFM binding's decode glue (BlackwellCpuFallback.java:50-79) ----
 * Path: backend/blackwell/aljabr-kernel-blackwell/src/main/java/tech/kayys/
 * aljabr/blackwell/binding/BlackwellCpuFallback.java.  rmsNorm: sequential
 * float sum of squares, rms = (float) Math.sqrt(sum / N + eps),
 * out = (x / rms) * w.  siluFfn: g / (1 + (float) Math.exp(-g)) * u. */
void orc_rmsnorm_binding(const float* x, const float* w, float* out, int n, float eps) {
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += x[i] * x[i];
    const float rms = (float)sqrt((double)(sum / (float)n + eps));
    for (int i = 0; i < n; i++) out[i] = (x[i] / rms) * w[i];
}
void orc_silu_ffn_binding(const float* gate, const float* up, float* out, int n) {
    for (int i = 0; i < n; i++) {
        const float g = gate[i];
        const float silu = g / (1.0f + (float)exp(-(double)g));
        out[i] = silu * up[i];
    }
}

/* ------------------------------------------------------------------------ */
/* Row parallelism: rows split into 2 chunks per thread, chunks pulled from a
 * shared counter (RT/GgufParallelConfig.java:14-15,56-73, GgufRows.java:133). */
typedef struct {
    int type, K, N, group, vector_order;
    const uint8_t* w; const float* absmax; const float* x; const float* bias;
    float* y; double* y64;
    int chunks; int next; pthread_mutex_t lock;
} job_t;

static float nf4_row_dot(const uint8_t* codes, const float* absmax, const float* x, int K, int group, int64_t row) {
    /* Dequantise the row exactly as DK:84-102 does for the flat tensor
     * (element e = row*K + k: nibble (e & 1 ? low : high) of byte e >> 1,
     * scale absmax[(e >> 1) * 2 / group]), then an 8-lane FMA dot with a
     * left-to-right lane sum -- the shape of a SIMD cblas_sgemv row, which
     * is what AccelOps.linear calls (closed, macOS-only; parity unpinned).
     * A plain sequential fp32 sum would itself drift past 1e-3 relative
     * error on K = 14336 rows with cancellation. */
    float acc[VLANES] = {0};
    int64_t base = row * (int64_t)K;
    for (int k = 0; k < K; k++) {
        int64_t e = base + k;
        int b = codes[e >> 1];
        int code = (e & 1) ? (b & 15) : ((b >> 4) & 15);
        float w = NF4_TABLE[code] * absmax[((e >> 1) * 2) / group];
        acc[k % VLANES] = fmaf(w, x[k], acc[k % VLANES]);
    }
    float s = 0.0f;
    for (int l = 0; l < VLANES; l++) s += acc[l];
    return s;
}

static double f64_row_dot(const job_t* j, int64_t row) {
    int K = j->K;
    double s = 0.0;
    if (j->type == ORC_Q4_0) {
        const uint8_t* r = j->w + row * (int64_t)(K / 32) * 18;
        for (int b = 0; b < K / 32; b++) {
            double d = orc_f16_to_f32(le16(r + b * 18));
            for (int t = 0; t < 16; t++) {
                int q = r[b * 18 + 2 + t];
                s += d * ((q & 15) - 8) * (double)j->x[b * 32 + t];
                s += d * ((q >> 4) - 8) * (double)j->x[b * 32 + 16 + t];
            }
        }
    } else if (j->type == ORC_Q8_0) {
        const uint8_t* r = j->w + row * (int64_t)(K / 32) * 34;
        for (int b = 0; b < K / 32; b++) {
            double d = orc_f16_to_f32(le16(r + b * 34));
            for (int t = 0; t < 32; t++) s += d * (int8_t)r[b * 34 + 2 + t] * (double)j->x[b * 32 + t];
        }
    } else if (j->type == ORC_Q4_K || j->type == ORC_Q6_K) {
        const int bb = j->type == ORC_Q4_K ? 144 : 210;
        double vals[256];
        for (int b = 0; b < K / 256; b++) {
            orc_dequantize_k_row(j->type, j->w + row * (int64_t)(K / 256) * bb + (int64_t)b * bb, 256, vals);
            for (int e = 0; e < 256; e++) s += vals[e] * (double)j->x[b * 256 + e];
        }
    } else {
        int64_t base = row * (int64_t)K;
        for (int k = 0; k < K; k++) {
            int64_t e = base + k;
            int b = j->w[e >> 1];
            int code = (e & 1) ? (b & 15) : ((b >> 4) & 15);
            s += (double)NF4_TABLE[code] * (double)j->absmax[((e >> 1) * 2) / j->group] * (double)j->x[k];
        }
    }
    return s;
}

static void* worker(void* arg) {
    job_t* j = (job_t*)arg;
    for (;;) {
        pthread_mutex_lock(&j->lock);
        int c = j->next++;
        pthread_mutex_unlock(&j->lock);
        if (c >= j->chunks) break;
        int64_t r0 = (int64_t)j->N * c / j->chunks, r1 = (int64_t)j->N * (c + 1) / j->chunks;
        for (int64_t r = r0; r < r1; r++) {
            if (j->y64) { j->y64[r] = f64_row_dot(j, r); continue; }
            float v;
            if (j->type == ORC_Q4_0) v = orc_dot_row_q4_0(j->w + r * (int64_t)(j->K / 32) * 18, j->K, j->x);
            else if (j->type == ORC_Q4_0_PREPARED)
                v = orc_dot_row_q4_0_prepared(j->w + r * (int64_t)(j->K / 32) * 18, j->K, j->x);
            else if (j->type == ORC_Q4_K) v = orc_dot_row_q4_k(j->w + r * (int64_t)(j->K / 256) * 144, j->K, j->x);
            else if (j->type == ORC_Q6_K) v = orc_dot_row_q6_k(j->w + r * (int64_t)(j->K / 256) * 210, j->K, j->x);
            else if (j->type == ORC_Q8_0)
                v = j->vector_order ? orc_dot_row_q8_0_vector(j->w + r * (int64_t)(j->K / 32) * 34, j->K, j->x)
                                    : orc_dot_row_q8_0_scalar(j->w + r * (int64_t)(j->K / 32) * 34, j->K, j->x);
            else {
                v = nf4_row_dot(j->w, j->absmax, j->x, j->K, j->group, r);
                if (j->bias) v += j->bias[r];
            }
            j->y[r] = v;
        }
    }
    return NULL;
}

static void run_job(job_t* j, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    j->chunks = threads == 1 ? 1 : threads * 2;
    if (j->chunks > j->N) j->chunks = j->N > 0 ? j->N : 1;
    j->next = 0;
    pthread_mutex_init(&j->lock, NULL);
    if (threads == 1) { worker(j); pthread_mutex_destroy(&j->lock); return; }
    pthread_t tid[256];
    for (int t = 0; t < threads; t++) pthread_create(&tid[t], NULL, worker, j);
    for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    pthread_mutex_destroy(&j->lock);
}

void orc_matvec_q4_0(const uint8_t* w, const float* x, float* y, int K, int N, int threads) {
    job_t j; memset(&j, 0, sizeof j);
    j.type = ORC_Q4_0; j.K = K; j.N = N; j.w = w; j.x = x; j.y = y;
    run_job(&j, threads);
}

void orc_matvec_q4_0_prepared(const uint8_t* w, const float* x, float* y, int K, int N, int threads) {
    job_t j; memset(&j, 0, sizeof j);
    j.type = ORC_Q4_0_PREPARED; j.K = K; j.N = N; j.w = w; j.x = x; j.y = y;
    run_job(&j, threads);
}

void orc_matvec_q8_0(const uint8_t* w, const float* x, float* y, int K, int N, int vector_order, int threads) {
    job_t j; memset(&j, 0, sizeof j);
    j.type = ORC_Q8_0; j.K = K; j.N = N; j.w = w; j.x = x; j.y = y; j.vector_order = vector_order;
    run_job(&j, threads);
}

void orc_matvec_k(int type, const uint8_t* w, const float* x, float* y, int K, int N, int threads) {
    job_t j; memset(&j, 0, sizeof j);
    j.type = type; j.K = K; j.N = N; j.w = w; j.x = x; j.y = y;
    run_job(&j, threads);
}

void orc_matvec_nf4(const uint8_t* codes, const float* absmax, const float* x, float* y,
                    int K, int N, int group_size, const float* bias, int threads) {
    job_t j; memset(&j, 0, sizeof j);
    j.type = ORC_NF4; j.K = K; j.N = N; j.w = codes; j.absmax = absmax; j.x = x; j.y = y;
    j.group = group_size; j.bias = bias;
    run_job(&j, threads);
}

void orc_matvec_f64(int type, const void* w, const float* absmax, const float* x, double* y,
                    int K, int N, int group_size, int threads) {
    job_t j; memset(&j, 0, sizeof j);
    j.type = type; j.K = K; j.N = N; j.w = (const uint8_t*)w; j.absmax = absmax; j.x = x;
    j.y64 = y; j.group = group_size;
    run_job(&j, threads);
}

/* ------------------------------------------------------------------------ */
float orc_vec_dot(const float* a, const float* b, int len) {   /* VO:43-55 */
    float acc[VLANES] = {0};
    int i = 0, bound = len - len % VLANES;
    for (; i < bound; i += VLANES)
        for (int l = 0; l < VLANES; l++) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float r = 0.0f;
    for (int l = 0; l < VLANES; l++) r += acc[l];
    for (; i < len; i++) r += a[i] * b[i];
    return r;
}

void orc_softmax(float* a, int len) {   /* VO:302-317 */
    float max = a[0];
    for (int i = 1; i < len; i++) if (a[i] > max) max = a[i];
    float sum = 0.0f;
    for (int i = 0; i < len; i++) {
        a[i] = (float)exp((double)(a[i] - max));
        sum += a[i];
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < len; i++) a[i] *= inv;
}

void orc_gqa_decode_attention(const float* q, float* out, float* scores,
                              const float* k_cache, const float* v_cache, int stride,
                              int kv_heads, int q_heads, int head_dim,
                              int seq_len, int start_pos, float scale) {   /* AT:70-106 */
    memset(out, 0, sizeof(float) * (size_t)q_heads * head_dim);
    int active = seq_len - start_pos;
    for (int head = 0; head < q_heads; head++) {
        int kv_head = head / (q_heads / kv_heads);
        const float* qh = q + (size_t)head * head_dim;
        for (int p = start_pos; p < seq_len; p++)
            scores[p - start_pos] = orc_vec_dot(qh, k_cache + (size_t)p * stride + (size_t)kv_head * head_dim, head_dim) * scale;
        orc_softmax(scores, active);
        float* oh = out + (size_t)head * head_dim;
        for (int p = start_pos; p < seq_len; p++) {
            const float* vr = v_cache + (size_t)p * stride + (size_t)kv_head * head_dim;
            float s = scores[p - start_pos];
            for (int i = 0; i < head_dim; i++) oh[i] = oh[i] + vr[i] * s;   /* VO:165-174 */
        }
    }
}

void orc_prefill_attention(float* out, const float* q, const float* k, const float* v, float* scores, int tokens,
                           int q_heads, int kv_heads, int head_dim, float scale, int window, int kv_stride) {
    for (int t = 0; t < tokens; t++) {                                        /* PA:44-82 */
        int start = window > 0 ? (t - window + 1 > 0 ? t - window + 1 : 0) : 0;
        int end = t;
        int active = end - start + 1;
        for (int head = 0; head < q_heads; head++) {
            int kv_head = head / (q_heads / kv_heads);
            const float* qh = q + (size_t)t * q_heads * head_dim + (size_t)head * head_dim;
            for (int p = start; p <= end; p++) {
                const float* kr = k + (size_t)p * kv_stride + (size_t)kv_head * head_dim;
                float dot = 0.0f;
                for (int d = 0; d < head_dim; d++) dot += qh[d] * kr[d];
                scores[p - start] = dot * scale;
            }
            orc_softmax(scores, active);
            float* oh = out + (size_t)t * q_heads * head_dim + (size_t)head * head_dim;
            for (int d = 0; d < head_dim; d++) oh[d] = 0.0f;
            for (int p = start; p <= end; p++) {
                float w = scores[p - start];
                const float* vr = v + (size_t)p * kv_stride + (size_t)kv_head * head_dim;
                for (int d = 0; d < head_dim; d++) oh[d] += w * vr[d];
            }
        }
    }
}

void orc_fa4_attention(float* out, const float* q, const float* k, const float* v, float* scores, int B, int T,
                       int S, int H, int H_kv, int D, float scale, int causal, float soft_cap) {
    int group = H / H_kv;                                                     /* FA:46-104 */
    int off = S - T > 0 ? S - T : 0;
    for (int b = 0; b < B; b++)
        for (int h = 0; h < H; h++) {
            int hk = h / group;
            for (int t = 0; t < T; t++) {
                float mx = -INFINITY;
                const float* qr = q + ((size_t)(b * T * H + t * H + h)) * D;
                for (int s = 0; s < S; s++) {
                    if (causal && s > off + t) { scores[s] = -INFINITY; continue; }
                    const float* kr = k + ((size_t)(b * S * H_kv + s * H_kv + hk)) * D;
                    float dot = 0.0f;
                    for (int d = 0; d < D; d++) dot += qr[d] * kr[d];
                    float score = dot * scale;
                    if (soft_cap > 0.0f) score = (float)(tanh((double)(score / soft_cap)) * (double)soft_cap);
                    scores[s] = score;
                    if (scores[s] > mx) mx = scores[s];
                }
                float sum = 0.0f;
                for (int s = 0; s < S; s++) {
                    if (!causal || s <= off + t) {
                        scores[s] = (float)exp((double)(scores[s] - mx));
                        sum += scores[s];
                    } else {
                        scores[s] = 0.0f;
                    }
                }
                if (sum > 0.0f)
                    for (int s = 0; s < S; s++) scores[s] /= sum;
                float* orow = out + ((size_t)(b * T * H + t * H + h)) * D;
                for (int d = 0; d < D; d++) {
                    float acc = 0.0f;
                    for (int s = 0; s < S; s++)
                        acc += scores[s] * v[((size_t)(b * S * H_kv + s * H_kv + hk)) * D + d];
                    orow[d] = acc;
                }
            }
        }
}

void orc_rms_norm(const float* x, const float* w, float* out, int len, float eps) {   /* VO:211-234 */
    float acc[VLANES] = {0};
    int i = 0, bound = len - len % VLANES;
    for (; i < bound; i += VLANES)
        for (int l = 0; l < VLANES; l++) acc[l] = fmaf(x[i + l], x[i + l], acc[l]);
    float ss = 0.0f;
    for (int l = 0; l < VLANES; l++) ss += acc[l];
    for (; i < len; i++) ss += x[i] * x[i];
    float scale = 1.0f / (float)sqrt((double)(ss / (float)len + eps));
    for (i = 0; i < len; i++) out[i] = x[i] * scale * w[i];
}

void orc_rope(float* x, int n_heads, int head_dim, int rotary_dim, int pos, float freq_base) {   /* VO:383-440 */
    int half = rotary_dim / 2;
    float table[2048];
    for (int i = 0; i < half; i++) {
        float expo = -2.0f * (float)i / (float)rotary_dim;
        float inv_freq = (float)pow((double)freq_base, (double)expo);
        float theta = ((float)pos * inv_freq) / 1.0f;
        table[i] = (float)cos((double)theta);
        table[half + i] = (float)sin((double)theta);
    }
    for (int h = 0; h < n_heads; h++) {
        float* b = x + (size_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            float c = table[i], s = table[half + i];
            float x0 = b[i], x1 = b[i + half];
            b[i] = x0 * c - x1 * s;
            b[i + half] = x0 * s + x1 * c;
        }
    }
}

void orc_swiglu(const float* gate, const float* up, float* dst, int len) {   /* VO:333-338 */
    for (int i = 0; i < len; i++) {
        float g = gate[i] / (1.0f + (float)exp(-(double)gate[i]));
        dst[i] = g * up[i];
    }
}

/* ------------------------------------------------------------------------ */
static int64_t typed_row_bytes(int type, int K) {
    switch (type) {
        case ORC_Q4_0: return (int64_t)K / 32 * 18;
        case ORC_Q8_0: return (int64_t)K / 32 * 34;
        case ORC_Q4_K: return (int64_t)K / 256 * 144;
        case ORC_Q6_K: return (int64_t)K / 256 * 210;
        default: return (int64_t)K / 2;
    }
}

/* y = W x with each row dotted in the reference's raw-row float order for
 * the tensor's GGUF type (GgufRawDot's q4_0 / q8_0 / q4K / q6K routes), or
 * AccelOps.linear's NF4 order. */
static void typed_rows(int type, const uint8_t* w, const float* absmax, const float* x, float* y, int K, int g,
                       int64_t r0, int64_t r1) {
    const int64_t rb = typed_row_bytes(type, K);
    for (int64_t r = r0; r < r1; r++) {
        const uint8_t* row = w + r * rb;
        switch (type) {
            case ORC_Q4_0: y[r] = orc_dot_row_q4_0(row, K, x); break;
            case ORC_Q8_0: y[r] = orc_dot_row_q8_0_scalar(row, K, x); break;
            case ORC_Q4_K: y[r] = orc_dot_row_q4_k(row, K, x); break;
            case ORC_Q6_K: y[r] = orc_dot_row_q6_k(row, K, x); break;
            default: y[r] = nf4_row_dot(w, absmax, x, K, g, r); break;
        }
    }
}

/* Host threads for the decode-step restatement's matvecs (each row is
 * computed by one thread in its own fixed order, so the result does not
 * depend on the count; only the checker's speed does). */
static int g_decode_threads = 1;
void orc_set_decode_threads(int threads) { g_decode_threads = threads < 1 ? 1 : (threads > 256 ? 256 : threads); }

typedef struct {
    int type, K, N, g;
    const uint8_t* w; const float* absmax; const float* x; float* y;
    int part, parts;
} typed_job_t;
static void* typed_worker(void* arg) {
    typed_job_t* j = (typed_job_t*)arg;
    typed_rows(j->type, j->w, j->absmax, j->x, j->y, j->K, j->g, (int64_t)j->N * j->part / j->parts,
               (int64_t)j->N * (j->part + 1) / j->parts);
    return NULL;
}
static void typed_matvec_seq(int type, const uint8_t* w, const float* absmax, const float* x, float* y, int K, int N,
                             int g) {
    const int parts = N >= 64 * g_decode_threads ? g_decode_threads : 1;
    if (parts == 1) {
        typed_rows(type, w, absmax, x, y, K, g, 0, N);
        return;
    }
    pthread_t tid[256];
    typed_job_t jobs[256];
    for (int p = 0; p < parts; p++) {
        jobs[p] = (typed_job_t){type, K, N, g, w, absmax, x, y, p, parts};
        pthread_create(&tid[p], NULL, typed_worker, &jobs[p]);
    }
    for (int p = 0; p < parts; p++) pthread_join(tid[p], NULL);
}

/* One GGUF row (`cols` values) as floats, in the reference's dequantiser
 * order: Q4_0 / Q8_0 as GgufBlockDequantizer (orc_dequantize_q4_0 / _q8_0),
 * Q4_K as GgufKBlockDequantizer.dequantizeQ4KBlock (:32-75: d1 = d * scale,
 * m1 = dmin * min, value = d1 * q - m1), Q6_K as dequantizeQ6KBlock
 * (:320-360: s = d * scale, value = s * (q - 32)). */
void orc_dequantize_row_ref(int type, const uint8_t* row, int cols, float* x) {
    if (type == ORC_Q4_0) {
        orc_dequantize_q4_0(row, x, cols);
    } else if (type == ORC_Q8_0) {
        orc_dequantize_q8_0(row, x, cols);
    } else if (type == ORC_Q4_K) {
        for (int b = 0; b < cols / 256; b++) {
            const uint8_t* blk = row + (int64_t)b * 144;
            const float d = orc_f16_to_f32(le16(blk)), dmin = orc_f16_to_f32(le16(blk + 2));
            for (int e = 0; e < 256; e++) {
                const int j = e / 64, t = e % 64, sb = 2 * j + (t >= 32);
                const int byte = blk[16 + 32 * j + (t & 31)];
                const int q = t < 32 ? (byte & 15) : (byte >> 4);
                int sc, mn;
                q4k_scale_min(blk + 4, sb, &sc, &mn);
                const float d1 = d * (float)sc, m1 = dmin * (float)mn;
                x[b * 256 + e] = d1 * (float)q - m1;
            }
        }
    } else if (type == ORC_Q6_K) {
        for (int b = 0; b < cols / 256; b++) {
            const uint8_t* blk = row + (int64_t)b * 210;
            const float d = orc_f16_to_f32(le16(blk + 208));
            for (int e = 0; e < 256; e++) {
                const int h = e / 128, w2 = e % 128, k = w2 / 32, i = w2 % 32;
                const int lo = blk[64 * h + 32 * (k & 1) + i];
                const int hb = blk[128 + 32 * h + i];
                const int q = (((k >> 1) ? (lo >> 4) : (lo & 15)) | (((hb >> (2 * k)) & 3) << 4)) - 32;
                const float s = d * (float)(int8_t)blk[192 + 8 * h + 2 * k + i / 16];
                x[b * 256 + e] = s * (float)q;
            }
        }
    }
}

/* Row `token` of an embedding table as floats: orc_dequantize_row_ref for the
 * GGUF types, DequantizationKernel.dequantizeNf4 for NF4. */
static void typed_embed_row(int type, const uint8_t* w, const float* absmax, int token, int H, int g, float* x) {
    if (type != ORC_NF4) {
        orc_dequantize_row_ref(type, w + (int64_t)token * typed_row_bytes(type, H), H, x);
        return;
    }
    const int64_t base = (int64_t)token * H;
    for (int k2 = 0; k2 < H; k2++) {
        const int64_t e = base + k2;
        const int bb = w[e >> 1];
        const int code = (e & 1) ? (bb & 15) : ((bb >> 4) & 15);
        x[k2] = NF4_TABLE[code] * absmax[((e >> 1) * 2) / g];
    }
}

void orc_decode_step_typed(const orc_llama_cfg* c, const uint8_t* const* codes, const int* types,
                           const float* const* absmax, const float* norms, void* k_cache_v, void* v_cache_v,
                           int kv_bf16, int token, int pos, float* x_out, float* logits) {
    int H = c->hidden, D = c->head_dim, Hq = c->q_heads, Hkv = c->kv_heads, F = c->ffn;
    int QD = Hq * D, KVD = Hkv * D, L = c->layers, g = c->group;
    float* x = (float*)calloc((size_t)H, 4);
    float* xb = (float*)calloc((size_t)(H > QD ? H : QD), 4);
    float* q = (float*)calloc((size_t)QD, 4);
    float* k = (float*)calloc((size_t)KVD, 4);
    float* v = (float*)calloc((size_t)KVD, 4);
    float* att = (float*)calloc((size_t)QD, 4);
    float* gate = (float*)calloc((size_t)F, 4);
    float* up = (float*)calloc((size_t)F, 4);
    float* hb = (float*)calloc((size_t)F, 4);
    float* scores = (float*)calloc((size_t)(pos + 1), 4);
    float* kf = (float*)calloc((size_t)(pos + 1) * KVD, 4);
    float* vf = (float*)calloc((size_t)(pos + 1) * KVD, 4);

    /* embedding row `token` (tensor 7*L) */
    typed_embed_row(types[7 * L], codes[7 * L], absmax[7 * L], token, H, g, x);
    float scale = (float)(1.0 / sqrt((double)D));                           /* DP:368-377 */
    for (int l = 0; l < L; l++) {
        const uint8_t* const* cw = codes + 7 * l;
        const float* const* aw = absmax + 7 * l;
        const int* tw = types + 7 * l;
        orc_rms_norm(x, norms + (size_t)l * 2 * H, xb, H, c->eps);             /* DP:305 */
        typed_matvec_seq(tw[0], cw[0], aw[0], xb, q, H, QD, g);                           /* DP:309 */
        typed_matvec_seq(tw[1], cw[1], aw[1], xb, k, H, KVD, g);
        typed_matvec_seq(tw[2], cw[2], aw[2], xb, v, H, KVD, g);
        orc_rope(q, Hq, D, D, pos, c->rope_theta);                               /* DP:333 */
        orc_rope(k, Hkv, D, D, pos, c->rope_theta);                              /* DP:360 */
        size_t lbase = (size_t)l * c->max_ctx * KVD;
        if (kv_bf16) {                                                           /* DP:362 */
            uint16_t* kc = (uint16_t*)k_cache_v;
            uint16_t* vc = (uint16_t*)v_cache_v;
            for (int i = 0; i < KVD; i++) {
                kc[lbase + (size_t)pos * KVD + i] = orc_f32_to_bf16_rne(k[i]);
                vc[lbase + (size_t)pos * KVD + i] = orc_f32_to_bf16_rne(v[i]);
            }
            for (size_t i = 0; i < (size_t)(pos + 1) * KVD; i++) {
                kf[i] = bf16_to_f32(kc[lbase + i]);
                vf[i] = bf16_to_f32(vc[lbase + i]);
            }
        } else {
            float* kc = (float*)k_cache_v;
            float* vc = (float*)v_cache_v;
            memcpy(kc + lbase + (size_t)pos * KVD, k, sizeof(float) * KVD);
            memcpy(vc + lbase + (size_t)pos * KVD, v, sizeof(float) * KVD);
            memcpy(kf, kc + lbase, sizeof(float) * (size_t)(pos + 1) * KVD);
            memcpy(vf, vc + lbase, sizeof(float) * (size_t)(pos + 1) * KVD);
        }
        orc_gqa_decode_attention(q, att, scores, kf, vf, KVD, Hkv, Hq, D, pos + 1, 0, scale);   /* DP:386 */
        typed_matvec_seq(tw[3], cw[3], aw[3], att, xb, QD, H, g);                         /* DP:475 */
        for (int i = 0; i < H; i++) x[i] += xb[i];                               /* DP:481 */
        orc_rms_norm(x, norms + (size_t)l * 2 * H + H, xb, H, c->eps);           /* DP:485 */
        typed_matvec_seq(tw[4], cw[4], aw[4], xb, gate, H, F, g);                         /* DP:492 */
        typed_matvec_seq(tw[5], cw[5], aw[5], xb, up, H, F, g);
        orc_swiglu(gate, up, hb, F);                                             /* DP:497 */
        typed_matvec_seq(tw[6], cw[6], aw[6], hb, xb, F, H, g);                           /* DP:504 */
        for (int i = 0; i < H; i++) x[i] += xb[i];                               /* DP:511 */
    }
    memcpy(x_out, x, sizeof(float) * H);
    if (logits) {
        orc_rms_norm(x, norms + (size_t)L * 2 * H, xb, H, c->eps);
        typed_matvec_seq(types[7 * L + 1], codes[7 * L + 1], absmax[7 * L + 1], xb, logits, H, c->vocab, g);
    }
    free(x); free(xb); free(q); free(k); free(v); free(att); free(gate); free(up); free(hb);
    free(scores); free(kf); free(vf);
}

void orc_decode_step_nf4(const orc_llama_cfg* c, const uint8_t* const* codes, const float* const* absmax,
                         const float* norms, void* k_cache_v, void* v_cache_v, int kv_bf16,
                         int token, int pos, float* x_out, float* logits) {
    const int n = 7 * c->layers + 2;
    int* types = (int*)malloc(sizeof(int) * (size_t)n);
    for (int i = 0; i < n; i++) types[i] = ORC_NF4;
    orc_decode_step_typed(c, codes, types, absmax, norms, k_cache_v, v_cache_v, kv_bf16, token, pos, x_out, logits);
    free(types);
}
