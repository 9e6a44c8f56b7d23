"""Generate ``known_answers.json``: the reference's own known-answer tests for
the quantized decode path, restated as data.

The Java reference cannot run in this container (no JDK), so each fixture
below is transcribed from the reference test that holds it: the block bytes
the test writes, the activation it feeds, and the value it asserts.  Where
the Java test asserts against a formula of its own (``referenceQ4_0``,
``referencePreparedQ8``), the formula is evaluated here in float32 the same
way the test does and recorded with the test's tolerance.  Paths are relative
to the reference project root.

Run:  python tests/golden/make_golden.py   (writes tests/golden/known_answers.json)
"""
from __future__ import annotations

import json
import os

import numpy as np

RT_TEST = "engine/gguf/aljabr-gguf-core/src/test/java/tech/kayys/aljabr/gguf/runtime"
JB_TEST = "engine/gguf/aljabr-gguf-java/src/test/java/tech/kayys/aljabr/gguf/javabackend"
f32 = np.float32


def q4_block(d_bits: int, code_bytes) -> list:
    code_bytes = list(code_bytes)
    if len(code_bytes) == 1:
        code_bytes = code_bytes * 16
    return [d_bits & 0xFF, d_bits >> 8] + [b & 0xFF for b in code_bytes]


def q8_block(d_bits: int, quants) -> list:
    quants = list(quants)
    if len(quants) == 1:
        quants = quants * 32
    return [d_bits & 0xFF, d_bits >> 8] + [q & 0xFF for q in quants]


def ones(n):
    return [1.0] * n


def ramp(n):                      # GgufFx.java:51-57
    return [float(i + 1) for i in range(n)]


def patterned(n):                 # GgufQ32RawTest.java:213-219, GgufQ8Test.java:72-74
    return [float(f32(i % 23 - 11) * f32(0.0625)) for i in range(n)]


def main():
    fx = []

    # --- Q4_0 -----------------------------------------------------------
    fx.append(dict(
        name="q4_0_rowdot_ones", kind="q4_0_matvec",
        source=f"{RT_TEST}/GgufQ32Test.java:18-42",
        K=32, N=2,
        weights=q4_block(0x3C00, [0x98]) + q4_block(0x3C00, [0xA9]),
        x=ones(32), expected=[16.0, 48.0], tol=0.0))
    fx.append(dict(
        name="q4_0_dequant_row0", kind="q4_0_dequant",
        source=f"{RT_TEST}/GgufQ32Test.java:26-31",
        numel=32, weights=q4_block(0x3C00, [0x98]),
        expected=[0.0] * 16 + [1.0] * 16, tol=0.0))
    # GgufQ32Q4LaneTest.java:16-34 with GgufNibFx.java:13-25 lane-order bytes
    lane_bytes = [(i & 0x0F) | ((15 - i) << 4) for i in range(16)]
    fx.append(dict(
        name="q4_0_lane_order_ramp", kind="q4_0_matvec",
        source=f"{RT_TEST}/GgufQ32Q4LaneTest.java:16-34",
        K=32, N=1, weights=q4_block(0x3C00, lane_bytes), x=ramp(32), expected=[-264.0], tol=0.0))
    fx.append(dict(
        name="q4_0_lane_order_dequant", kind="q4_0_dequant",
        source=f"{RT_TEST}/GgufQ32Q4Fx.java:39-45",
        numel=32, weights=q4_block(0x3C00, lane_bytes),
        expected=[float((i & 0x0F) - 8) for i in range(16)] + [float((15 - i) - 8) for i in range(16)],
        tol=0.0))
    # GgufQ32RawTest.java:72-100: five blocks, unrolled loop plus a tail block
    half = [0x3C00, 0x4000, 0xBC00, 0x3800, 0x4200]
    scales = [1.0, 2.0, -1.0, 0.5, 3.0]
    packed = [0x21, 0x43, 0x65, 0x87, 0xA9]
    vec = patterned(5 * 32)
    s = f32(0.0)
    for b in range(5):                                 # referenceQ4_0 :221-236
        lo, hi = packed[b] & 0x0F, packed[b] >> 4
        for i in range(16):
            s = f32(s + f32(f32(scales[b]) * f32(lo - 8)) * f32(vec[b * 32 + i]))
            s = f32(s + f32(f32(scales[b]) * f32(hi - 8)) * f32(vec[b * 32 + 16 + i]))
    w = []
    for b in range(5):
        w += q4_block(half[b], [packed[b]])
    fx.append(dict(
        name="q4_0_five_blocks_patterned", kind="q4_0_matvec",
        source=f"{RT_TEST}/GgufQ32RawTest.java:72-100",
        K=160, N=1, weights=w, x=vec, expected=[float(s)], tol=1e-3))
    # GgufQ32TailTest.java:46-86: four one-block rows, packed 0x21+row, ones
    w, exp = [], []
    for row in range(4):
        p = 0x21 + row
        w += q4_block(0x3C00, [p])
        exp.append(float(16 * ((p & 0x0F) - 8) + 16 * ((p >> 4) - 8)))
    fx.append(dict(
        name="q4_0_tiny_rows_ones", kind="q4_0_matvec",
        source=f"{RT_TEST}/GgufQ32TailTest.java:46-86",
        K=32, N=4, weights=w, x=ones(32), expected=exp, tol=0.0))

    # --- Q8_0 -----------------------------------------------------------
    fx.append(dict(
        name="q8_0_rowdot_ones", kind="q8_0_matvec",
        source=f"{RT_TEST}/GgufQ8Test.java:21-45",
        K=32, N=2, weights=q8_block(0x3C00, [1]) + q8_block(0x3C00, [2]),
        x=ones(32), expected=[32.0, 64.0], tol=0.0))
    ramp_neg = [(-16 + i) for i in range(32)]          # GgufQ8Fx.java:26-31, start -16
    ramp_pos = [(16 - i) for i in range(32)]           # start 16
    fx.append(dict(
        name="q8_0_signed_lane_order_ramp", kind="q8_0_matvec",
        source=f"{RT_TEST}/GgufQ8RawTest.java:80-100",
        K=32, N=2, weights=q8_block(0x3C00, ramp_neg) + q8_block(0x3C00, ramp_pos),
        x=ramp(32), expected=[2464.0, -2464.0], tol=0.0))
    # GgufQ8Test.java:60-80: five blocks, q8Pattern(seed, i) = (byte)(seed + 37 i)
    q8s = [1.0, 2.0, -1.0, 0.5, -1.75]
    q8h = [0x3C00, 0x4000, 0xBC00, 0x3800, 0xBF00]
    seeds = [17, 43, 71, 103, 149]
    vec = patterned(5 * 32)

    def q8pat(seed, i):
        v = (seed + i * 37) & 0xFF
        return v - 256 if v >= 128 else v

    s = f32(0.0)
    w = []
    for b in range(5):                                 # referencePreparedQ8 :256-268
        w += q8_block(q8h[b], [q8pat(seeds[b], i) for i in range(32)])
        for i in range(32):
            s = f32(s + f32(f32(q8s[b]) * f32(q8pat(seeds[b], i))) * f32(vec[b * 32 + i]))
    fx.append(dict(
        name="q8_0_five_blocks_patterned", kind="q8_0_matvec",
        source=f"{RT_TEST}/GgufQ8Test.java:60-80",
        K=160, N=1, weights=w, x=vec, expected=[float(s)], tol=1e-3))

    # --- fp16 scale decoding ---------------------------------------------
    fx.append(dict(
        name="f16_special_values", kind="f16",
        source=f"{RT_TEST}/GgufF16SpecialTest.java:14-36",
        bits=[0x0000, 0x8000, 0x7C00, 0xFC00, 0x0001, 0x7E00],
        expected_bits=[0x00000000, 0x80000000, 0x7F800000, 0xFF800000, 0x33800000, "nan"]))

    # --- decode attention --------------------------------------------------
    fx.append(dict(
        name="gqa_maps_query_heads_to_kv_heads", kind="attention",
        source=f"{JB_TEST}/GgufDecodeAttentionExecutionTest.java:14-28",
        q=[0.0] * 4, k=[0.0] * 4, v=[10.0, 100.0, 20.0, 200.0],
        stride=2, kv_heads=2, q_heads=4, head_dim=1, seq_len=2, start=0, scale=1.0,
        expected=[15.0, 15.0, 150.0, 150.0], tol=1e-6))
    fx.append(dict(
        name="gqa_sliding_window_start", kind="attention",
        source=f"{JB_TEST}/GgufDecodeAttentionExecutionTest.java:30-43",
        q=[0.0] * 2, k=[0.0] * 4, v=[10.0, 100.0, 20.0, 200.0],
        stride=2, kv_heads=2, q_heads=2, head_dim=1, seq_len=2, start=1, scale=1.0,
        expected=[20.0, 200.0], tol=1e-6))
    fx.append(dict(
        name="gqa_session_window_average", kind="attention",
        source=f"{JB_TEST}/GgufDecodeAttentionExecutionTest.java:44-66",
        q=[0.0], k=[0.0, 0.0, 0.0], v=[10.0, 20.0, 30.0],
        stride=1, kv_heads=1, q_heads=1, head_dim=1, seq_len=3, start=1, scale=1.0,
        expected=[25.0], tol=1e-6))

    # --- NF4 (table + nibble order; no reference test pins NF4 values) ------
    nf4 = [-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
           -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
           0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
           0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0]
    codes = [(2 * i) << 4 | (2 * i + 1) for i in range(8)]   # codes 0..15 in order
    fx.append(dict(
        name="nf4_table_high_nibble_first", kind="nf4_dequant",
        source="engine/safetensor/aljabr-safetensor-core/src/main/java/tech/kayys/aljabr/"
               "safetensor/core/tensor/DequantizationKernel.java:23-28,84-102",
        numel=16, group=8, codes=codes, absmax=[2.0, -0.5],
        expected=[float(f32(nf4[i]) * f32(2.0 if i < 8 else -0.5)) for i in range(16)], tol=0.0))

    # --- Q4_K / Q6_K (256-value super-blocks) -------------------------------
    def lane_packed(i):           # GgufQ4CalcFx.packedQuant / GgufQ6Fx.laneOrderLowBits
        low = i & 0x0F
        return low | ((15 - low) << 4)

    def q4k_block(with_mins):     # GgufQ4Fx.writeSimpleBlock / writeBlockWithAllScalesAndMins + lane-order quants
        dmin = 0x3800 if with_mins else 0
        scales = [1, 1, 1, 1, 2, 2, 2, 2, 0x21, 0x21, 0x21, 0x21] if with_mins else \
                 [1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1]
        return [0x00, 0x3C, dmin & 0xFF, dmin >> 8] + scales + [lane_packed(i) for i in range(128)]

    def q4k_expected_dot(x, with_mins):   # GgufQ4CalcFx.expectedDot, float32 accumulation
        acc = f32(0)
        for sb in range(0, 256, 64):
            qb = (sb // 64) * 32
            for i in range(32):
                low = (qb + i) & 0x0F
                high = 15 - low
                lv = f32(low - 1.0) if with_mins else f32(low)
                hv = f32(high - 1.0) if with_mins else f32(high)
                acc = f32(acc + lv * f32(x[sb + i]))
                acc = f32(acc + hv * f32(x[sb + 32 + i]))
        return float(acc)

    for with_mins, lines in ((False, "20-43"), (True, "45-68")):
        fx.append(dict(
            name=f"q4_k_lane_order_{'mins' if with_mins else 'no_mins'}_ramp", kind="k_matvec",
            source=f"{RT_TEST}/GgufQ4KRawTest.java:{lines}, GgufQ4Fx.java, GgufQ4CalcFx.java",
            type=12, K=256, N=1, weights=q4k_block(with_mins), x=ramp(256),
            expected=[q4k_expected_dot(ramp(256), with_mins)], tol=0.0))

    def q6k_block(low, high, scale):      # GgufQ6Fx.writeBlock
        return [low] * 128 + [high] * 64 + [scale & 0xFF] * 16 + [0x00, 0x3C]

    fx.append(dict(
        name="q6_k_uniform_blocks_ones", kind="k_matvec",
        source=f"{RT_TEST}/GgufQ6KRawTest.java:20-45, GgufQ6Fx.java",
        type=14, K=256, N=2, weights=q6k_block(0x11, 0xAA, 1) + q6k_block(0x22, 0xAA, 1), x=ones(256),
        expected=[256.0, 512.0], tol=0.0))

    def q6_high(i):               # GgufQ6Fx.laneOrderHighBits
        return (i * 53 + 0xA7) & 0xFF

    q6_lane = [lane_packed(i) for i in range(128)] + [q6_high(i) for i in range(64)] + [1] * 16 + [0x00, 0x3C]

    def q6k_expected_dot(x):      # GgufQ6LaneFx.expectedDot, float32 accumulation
        acc = f32(0)
        for sb in range(0, 256, 128):
            lb, hb = (sb // 128) * 64, (sb // 128) * 32
            for i in range(32):
                a, c, h = lane_packed(lb + i), lane_packed(lb + 32 + i), q6_high(hb + i)
                vals = [((a & 15) | ((h & 3) << 4)) - 32, ((c & 15) | (((h >> 2) & 3) << 4)) - 32,
                        ((a >> 4) | (((h >> 4) & 3) << 4)) - 32, ((c >> 4) | (((h >> 6) & 3) << 4)) - 32]
                for q, off in zip(vals, (0, 32, 64, 96)):
                    acc = f32(acc + f32(q) * f32(x[sb + off + i]))
        return float(acc)

    fx.append(dict(
        name="q6_k_lane_order_ramp", kind="k_matvec",
        source=f"{RT_TEST}/GgufQ6KRawTest.java:47-75, GgufQ6Fx.java, GgufQ6LaneFx.java",
        type=14, K=256, N=2, weights=q6_lane + q6_lane, x=ramp(256),
        expected=[q6k_expected_dot(ramp(256))] * 2, tol=0.0))

    # K-quant row dequantisation (GgufKBlockDequantizer, the embedding-row path)
    fx.append(dict(
        name="q4_k_simple_block_dequant", kind="k_dequant",
        source=f"{RT_TEST}/GgufQ4KTest.java:17-35, GgufQ4Fx.java:13-24",
        type=12, K=256, weights=[0x00, 0x3C, 0x00, 0x00] + [1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1] + [0x21] * 128,
        expected=([1.0] * 32 + [2.0] * 32) * 4, tol=0.0))
    fx.append(dict(
        name="q6_k_uniform_block_dequant", kind="k_dequant",
        source=f"{RT_TEST}/GgufQ6KTest.java:18-32, GgufQ6Fx.java:13-28",
        type=14, K=256, weights=q6k_block(0x11, 0xAA, 1), expected=[1.0] * 256, tol=0.0))

    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "known_answers.json")
    with open(out, "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "fixtures": fx}, f, indent=1)
    print(f"wrote {len(fx)} fixtures to {out}")


if __name__ == "__main__":
    main()
