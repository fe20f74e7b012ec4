"""The reference's known-answer tests for its low-bit formats (src/metal/compute.rs:2384-2977),
as data: each case builds the same block bytes and input vector as the Rust test and keeps
its expected value and tolerance. Used by the oracle's CPU test and the GPU parity test."""
import numpy as np

Q2_K, Q3_K, IQ2_XXS, IQ2_XS, IQ3_XXS, IQ4_NL, IQ3_S, IQ4_XS = 10, 11, 16, 17, 18, 20, 21, 23
BLOCK = {Q2_K: (256, 84), Q3_K: (256, 110), IQ2_XXS: (256, 66), IQ2_XS: (256, 74),
         IQ3_XXS: (256, 98), IQ4_NL: (32, 18), IQ3_S: (256, 110), IQ4_XS: (256, 148)}
LOWBIT = tuple(BLOCK)


def f16le(v):
    return list(np.float16(v).view(np.uint16).tobytes())


def _case(name, wtype, rows, cols, block, x, expect, tol, cmp="abs"):
    return dict(name=name, type=wtype, rows=rows, cols=cols,
                raw=np.array(block, np.uint8), x=np.asarray(x, np.float32),
                expect=np.atleast_1d(np.asarray(expect, np.float64)), tol=tol, cmp=cmp)


def cases():
    out = []
    ones256, ones32 = np.ones(256), np.ones(32)
    # Q3_K (compute.rs:2384-2397, 2416-2434)
    b = [0] * 110
    b[108:110] = f16le(1.0)
    out.append(_case("q3_k_basic", Q3_K, 1, 256, b, ones256, 0.0, 1e-5))
    b = [0] * 110
    b[108:110] = f16le(0.5)
    b[96] = 0x01
    out.append(_case("q3_k_nonzero", Q3_K, 1, 256, b, ones256, -32.0, 1e-3))
    # Q2_K (:2458-2520)
    b = [0] * 84
    b[0:2] = f16le(1.0)
    out.append(_case("q2_k_basic", Q2_K, 1, 256, b, ones256, 0.0, 1e-5))
    b = [0] * 84
    b[0:2] = f16le(1.0)
    b[4] = 0x02
    b[20:24] = [0x55] * 4
    out.append(_case("q2_k_nonzero", Q2_K, 1, 256, b, ones256, 32.0, 1e-3))
    b = [0] * 84
    b[0:2] = f16le(1.0)
    b[2:4] = f16le(0.5)
    b[4] = 0x20
    out.append(_case("q2_k_with_min", Q2_K, 1, 256, b, ones256, -16.0, 1e-3))
    # IQ4_NL (:2565-2637, 2713-2726)
    b = [0] * 18
    b[0:2] = f16le(1.0)
    out.append(_case("iq4_nl_basic", IQ4_NL, 1, 32, b, ones32, -127.0 * 32, 1.0))
    b = [0] * 18
    b[0:2] = f16le(0.5)
    b[2] = 0xF8
    x = np.zeros(32)
    x[0:2] = 1.0
    out.append(_case("iq4_nl_lut_values", IQ4_NL, 1, 32, b, x, 0.5 * 114.0, 0.5))
    b = [0] * 36
    b[0:2] = f16le(1.0)
    b[2:18] = [0x88] * 16
    b[18:20] = f16le(2.0)
    b[20:36] = [0x88] * 16
    out.append(_case("iq4_nl_two_rows", IQ4_NL, 2, 32, b, ones32, [32.0, 64.0], 1.0))
    b = [0] * 18
    b[0:2] = f16le(1.0)
    b[2:18] = [0x88] * 16
    out.append(_case("iq4_nl_dispatch", IQ4_NL, 1, 32, b, ones32, 32.0, 1.0))
    # IQ4_XS (:2640-2700, 2728-2746)
    b = [0] * 148
    b[0:2] = f16le(1.0)
    b[20:148] = [0x88] * 128
    out.append(_case("iq4_xs_basic", IQ4_XS, 1, 256, b, ones256, -32.0 * 256, 10.0))
    b = [0] * 148
    b[0:2] = f16le(0.01)
    b[2:4] = [0xAA, 0xAA]
    for i in range(8):
        b[4 + 2 * i] = 0x11
    b[20:148] = [0x88] * 128
    out.append(_case("iq4_xs_positive_scale", IQ4_XS, 1, 256, b, ones256, 2.56, 0.5))
    # IQ3_XXS (:2748-2790)
    b = [0] * 98
    b[0:2] = f16le(1.0)
    out.append(_case("iq3_xxs_basic", IQ3_XXS, 1, 256, b, ones256, 256.0, 1.0))
    b[66:70] = [127, 0, 0, 0]
    out.append(_case("iq3_xxs_with_signs", IQ3_XXS, 1, 256, b, ones256, 240.0, 1.0))
    # IQ3_S (:2792-2845)
    b = [0] * 110
    b[0:2] = f16le(1.0)
    out.append(_case("iq3_s_basic", IQ3_S, 1, 256, b, ones256, 256.0, 1.0))
    b = [0] * 110
    b[0:2] = f16le(0.5)
    b[106:110] = [0x31] * 4
    out.append(_case("iq3_s_with_scale", IQ3_S, 1, 256, b, ones256, 640.0, 2.0))
    b = [0] * 110
    b[0:2] = f16le(1.0)
    b[74] = 0xFF
    out.append(_case("iq3_s_with_signs", IQ3_S, 1, 256, b, ones256, 240.0, 1.0))
    # IQ2_XXS (:2866-2910, 2961-2967)
    b = [0] * 66
    b[0:2] = [0x00, 0x3C]
    out.append(_case("iq2_xxs_basic", IQ2_XXS, 1, 256, b, ones256, 256.0, 1.0))
    b = [0] * 66
    b[0:2] = [0x00, 0x3C]
    b[6] = 0x7F
    out.append(_case("iq2_xxs_with_signs", IQ2_XXS, 1, 256, b, ones256, 0.0, 0.0, cmp="nonzero"))
    out.append(_case("iq2_xxs_dispatch", IQ2_XXS, 1, 256, [0] * 66, np.zeros(256), 0.0, 1e-6))
    # IQ2_XS (:2919-2950, 2970-2976)
    b = [0] * 74
    b[0:2] = [0x00, 0x3C]
    out.append(_case("iq2_xs_basic", IQ2_XS, 1, 256, b, ones256, 256.0, 1.0))
    b[66] = 0x5F
    out.append(_case("iq2_xs_with_scale", IQ2_XS, 1, 256, b, ones256, 256.0, 0.0, cmp="greater"))
    out.append(_case("iq2_xs_dispatch", IQ2_XS, 1, 256, [0] * 74, np.zeros(256), 0.0, 1e-6))
    return out


def check(case, y):
    y = np.asarray(y, np.float64)
    if case["cmp"] == "nonzero":
        return bool(np.all(np.abs(y) > 0.0))
    if case["cmp"] == "greater":
        return bool(np.all(y > case["expect"]))
    return bool(np.all(np.abs(y - case["expect"]) < case["tol"]))


def random_blocks(rng, wtype, rows, cols):
    """Random bytes of `rows` rows in the type's block layout, with every f16 scale set to a
    finite value of magnitude ~0.01-0.1 (random bytes there could be inf or NaN)."""
    bs, bb = BLOCK[wtype]
    nb = rows * (cols // bs)
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    d_at = {Q2_K: (0, 2), Q3_K: (108,), IQ4_XS: (0,), IQ4_NL: (0,), IQ3_XXS: (0,), IQ3_S: (0,),
            IQ2_XXS: (0,), IQ2_XS: (0,)}[wtype]
    for off in d_at:
        d = (rng.random(nb) * 0.09 + 0.01) * rng.choice([-1.0, 1.0], nb)
        raw[:, off:off + 2] = d.astype(np.float16).view(np.uint8).reshape(nb, 2)
    return raw.reshape(rows, -1)
