"""Device numerics of the overlay, restated in NumPy float32 (test oracle).

Reference semantics (Torch2RISCV-accelerator):
- fp32 add / mul: IEEE binary32, round to nearest even, no fused multiply-add,
  one rounding per step (`llm/fp32.py:1-20`; `llm/ref_model.py:151-163`).
  NumPy float32 arithmetic is exactly that for results in the normal range.
- EXP / RECIP / RSQRT: the SFU's table + one Newton step method
  (`llm/sfu.py:1-26`, tables `llm/sfu.py:43-58`, sequences `llm/sfu.py:69-114`),
  including its flush-to-zero of inputs and of the final exponent scaling.
- fixed-order fp32 sums over D = 16 lanes (`llm/ref_model.py:179-186`).
- int8 conversion: round to nearest even, saturate to +-127, NaN -> 0
  (`llm/ref_model.py:136-139`).
"""
import numpy as np

F = np.float32
U32 = np.uint32
D_LANES = 16                      # the KV260 overlay's array size (d16_100mhz_*), the reduction lane count
QNAN = U32(0x7FC00000)
PINF = U32(0x7F800000)
C127 = F(1 / 127)                 # F(1/127): `llm/ref_model.py:193`, `compile_layer.INV127`
LOG2E = F(1.4426950408889634)     # `llm/sfu.py:33`


def bits(x):
    return np.asarray(x, F).view(U32)


def flt(b):
    return np.asarray(b, U32).view(F)


# ----------------------------------------------------------------- SFU tables
_TABLES = None


def sfu_tables():
    """Segment starts T and slopes S of the SFU (`llm/sfu.py:43-58`): computed in
    float64, rounded once to float32. EXP/RECIP: 64 segments of [1, 2); RSQRT:
    64 segments of [1, 2) then 64 of [2, 4)."""
    global _TABLES
    if _TABLES is None:
        k = np.arange(64, dtype=np.float64)
        t_exp = 2.0 ** (k / 64)
        s_exp = 2.0 ** ((k + 1) / 64) - t_exp
        m = 1 + k / 64
        t_rec = 1 / m
        s_rec = 1 / (m + 1 / 64) - t_rec
        m2 = np.concatenate([1 + k / 64, 2 * (1 + k / 64)])
        step = np.concatenate([np.full(64, 1 / 64), np.full(64, 2 / 64)])
        t_rsq = 1 / np.sqrt(m2)
        s_rsq = 1 / np.sqrt(m2 + step) - t_rsq
        _TABLES = {"exp": (t_exp.astype(F), s_exp.astype(F)),
                   "recip": (t_rec.astype(F), s_rec.astype(F)),
                   "rsqrt": (t_rsq.astype(F), s_rsq.astype(F))}
    return _TABLES


def ftz(x):
    """Subnormal -> zero of the same sign (`llm/fp32.py:206-209`)."""
    b = bits(x)
    return flt(np.where(((b >> 23) & 0xFF) == 0, b & U32(0x80000000), b))


def ldexp_ftz(y, n):
    """y * 2^n by exponent addition, flushing below-normal results to a signed
    zero and overflow to a signed infinity (`llm/fp32.py:145-151`, `_pack`
    :53-60). y is a normal number, a zero, an infinity or a NaN."""
    b = bits(y).astype(np.int64)
    s, e, m = b >> 31, (b >> 23) & 0xFF, b & 0x7FFFFF
    ne = e + np.asarray(n, np.int64)
    out = (s << 31) | (np.clip(ne, 0, 255) << 23) | m
    out = np.where(ne < 1, s << 31, out)
    out = np.where(ne > 254, (s << 31) | (255 << 23), out)
    special = (e == 0) | (e == 255)
    out = np.where(special, np.where((e == 255) & (m != 0), int(QNAN), np.where(e == 0, s << 31, b)), out)
    return flt(out.astype(U32))


def _floor_int(v, lo, hi):
    with np.errstate(invalid="ignore"):
        f = np.floor(np.nan_to_num(np.asarray(v, np.float64), nan=0.0, posinf=hi, neginf=lo))
    return np.clip(f, lo, hi).astype(np.int64)


def sfu_exp(x):
    """EXP (`llm/sfu.py:69-82`): t = x*log2e, n = floor(t), f = t - n,
    u = 64f, i = floor(u), r = u - i, y = T[i] + r*S[i], y * 2^n; x >= 89 -> +inf,
    x <= -104 -> +0, NaN -> NaN."""
    T, S = sfu_tables()["exp"]
    x = ftz(x)
    with np.errstate(all="ignore"):
        t = (x * LOG2E).astype(F)
        n = _floor_int(t, -2**31, 2**31 - 1)
        f = (t - n.astype(F)).astype(F)
        u = (f * F(64)).astype(F)
        i = _floor_int(u, 0, 63)
        r = (u - i.astype(F)).astype(F)
        y = (T[i] + (r * S[i]).astype(F)).astype(F)
    res = bits(ldexp_ftz(y, np.clip(n, -300, 300)))
    with np.errstate(invalid="ignore"):
        xf = x.astype(np.float64)
    res = np.where(xf >= 89, PINF, np.where(xf <= -104, U32(0), res))
    return flt(np.where(np.isnan(xf), QNAN, res).astype(U32))


def _r17(frac):
    """(frac & 0x1FFFF) / 2^17, exact (`llm/sfu.py:64-66`)."""
    return ((frac & 0x1FFFF).astype(F) * F(2.0 ** -17)).astype(F)


def sfu_recip(x):
    """RECIP (`llm/sfu.py:85-96`): x = m*2^E, i = top 6 fraction bits,
    y0 = T[i] + r*S[i], y1 = y0*(2 - m*y0), result +-y1*2^-E; +-0 -> +-inf,
    +-inf -> +-0, NaN -> NaN."""
    T, S = sfu_tables()["recip"]
    b = bits(ftz(x)).astype(np.int64)
    s, e, frac = b >> 31, (b >> 23) & 0xFF, b & 0x7FFFFF
    i = frac >> 17
    m = flt((frac | 0x3F800000).astype(U32))
    with np.errstate(all="ignore"):
        y0 = (T[i] + (_r17(frac) * S[i]).astype(F)).astype(F)
        y1 = (y0 * (F(2.0) - (m * y0).astype(F)).astype(F)).astype(F)
    res = bits(ldexp_ftz(y1, 127 - e)).astype(np.int64) | (s << 31)
    res = np.where(e == 0, (s << 31) | 0x7F800000, res)
    res = np.where((e == 255) & (frac == 0), s << 31, res)
    res = np.where((e == 255) & (frac != 0), int(QNAN), res)
    return flt(res.astype(U32))


def sfu_rsqrt(x):
    """RSQRT (`llm/sfu.py:99-114`): x = m*2^E; odd E uses m' = 2m;
    j = 64*(E odd) + top 6 fraction bits; y0 = T[j] + r*S[j];
    y1 = y0*(1.5 - (m'*(y0*y0))*0.5); result y1*2^(-(E - odd)/2);
    NaN / negative -> NaN, +-0 -> +inf, +inf -> +0."""
    T, S = sfu_tables()["rsqrt"]
    b = bits(ftz(x)).astype(np.int64)
    s, e, frac = b >> 31, (b >> 23) & 0xFF, b & 0x7FFFFF
    E = e - 127
    odd = E & 1
    j = odd * 64 + (frac >> 17)
    m2 = flt((frac | ((127 + odd) << 23)).astype(U32))
    with np.errstate(all="ignore"):
        y0 = (T[j] + (_r17(frac) * S[j]).astype(F)).astype(F)
        d = (F(1.5) - ((m2 * (y0 * y0).astype(F)).astype(F) * F(0.5)).astype(F)).astype(F)
        y1 = (y0 * d).astype(F)
    res = bits(ldexp_ftz(y1, -((E - odd) // 2))).astype(np.int64)
    res = np.where(e == 0, int(PINF), res)
    res = np.where((s == 1) & (e != 0), int(QNAN), res)
    res = np.where((s == 0) & (e == 255) & (frac == 0), 0, res)
    res = np.where((e == 255) & (frac != 0), int(QNAN), res)
    return flt(res.astype(U32))


# ------------------------------------------------------ vector primitives
def to_i8(x):
    """fp32 -> int8, RNE, saturate +-127, NaN -> 0 (`llm/ref_model.py:136-139`)."""
    y = np.rint(np.asarray(x, F))
    return np.clip(np.nan_to_num(y, nan=0.0, posinf=127, neginf=-127), -127, 127).astype(np.int8)


def red_sum(v, d=D_LANES):
    """Fixed-order fp32 sum (`llm/ref_model.py:179-186`): zero-pad to a multiple
    of d, add the d-lane groups one after another, then a pairwise tree over the
    lanes (lane 2j + lane 2j+1 at every level)."""
    v = np.asarray(v, F)
    n = -v.size % d
    g = (np.concatenate([v, np.zeros(n, F)]) if n else v).reshape(-1, d)
    acc = g[0].copy()
    for row in g[1:]:
        acc = (acc + row).astype(F)
    while acc.size > 1:
        acc = (acc[0::2] + acc[1::2]).astype(F)
    return acc[0]


def red_sum_rows(v, d=D_LANES):
    """red_sum over the last axis of a 2-D array, row by row (vectorized)."""
    v = np.asarray(v, F)
    n = -v.shape[-1] % d
    if n:
        v = np.concatenate([v, np.zeros(v.shape[:-1] + (n,), F)], axis=-1)
    g = v.reshape(v.shape[0], -1, d)
    acc = g[:, 0].copy()
    for i in range(1, g.shape[1]):
        acc = (acc + g[:, i]).astype(F)
    while acc.shape[1] > 1:
        acc = (acc[:, 0::2] + acc[:, 1::2]).astype(F)
    return acc[:, 0]


def quant_act(x):
    """Per-token dynamic int8 (`llm/ref_model.py:191-196`): amax = max|x|,
    s_x = amax*F(1/127), inv = RECIP(s_x), xq = i8(x*inv). Rows of a 2-D x are
    independent tokens."""
    x = np.asarray(x, F)
    amax = np.max(np.abs(x), axis=-1, keepdims=True)
    s_x = (amax * C127).astype(F)
    inv = sfu_recip(s_x)
    with np.errstate(invalid="ignore"):
        return to_i8((x * inv).astype(F)), s_x[..., 0]


def linear(xq, s_x, wq, s_w):
    """W8A8 linear (`llm/ref_model.py:198-202`): acc = xq . W^T exact int32,
    y = (f32(acc)*s_w)*s_x. xq [.., K] int8, wq [N, K] int8."""
    acc = np.asarray(xq, np.int64) @ np.asarray(wq, np.int64).T
    y = (acc.astype(F) * np.asarray(s_w, F)).astype(F)
    return (y * np.asarray(s_x, F)[..., None]).astype(F), acc


def linear_f64(xq, s_x, wq_f64, s_w):
    """linear() with the weights as float64 (exact int dot products through
    BLAS, `llm/ref_model.py:164`); the fast form for large layers."""
    acc = (np.asarray(xq, np.float64) @ wq_f64.T).astype(np.int64)
    y = (acc.astype(F) * np.asarray(s_w, F)).astype(F)
    return (y * np.asarray(s_x, F)[..., None]).astype(F), acc


def rmsnorm(x, g, eps):
    """ss = red_sum(x*x), r = RSQRT(ss*F(1/n) + eps), y = (x*r)*g
    (`llm/ref_model.py:204-207`; `hf_generic.SaRMSNorm` :822-826 with the
    device's fixed-order sum). Rows of a 2-D x are normalized independently."""
    x = np.asarray(x, F)
    x2 = np.atleast_2d(x)
    ss = red_sum_rows((x2 * x2).astype(F))
    inv_n = F(1.0 / x2.shape[-1])
    r = sfu_rsqrt(((ss * inv_n).astype(F) + F(eps)).astype(F))
    y = (((x2 * r[:, None]).astype(F)) * np.asarray(g, F)).astype(F)
    return y.reshape(x.shape)


def swapneg(v):
    """(x0, x1) -> (-x1, x0) per pair (`llm/ref_model.py:212-213`)."""
    v = np.asarray(v, F)
    sw = np.empty_like(v)
    sw[..., 0::2], sw[..., 1::2] = -v[..., 1::2], v[..., 0::2]
    return sw


def rope(v, cos, sin):
    """(v*cos) + (swapneg(v)*sin), cos / sin already pair-repeated to v's
    shape (`llm/ref_model.py:209-214`)."""
    v = np.asarray(v, F)
    return ((v * cos).astype(F) + (swapneg(v) * sin).astype(F)).astype(F)


def silu_gate(g, u):
    """h = (g*RECIP(1 + EXP(g*-1)))*u (`llm/ref_model.py:249-250`)."""
    sig = sfu_recip((F(1) + sfu_exp((g * F(-1)).astype(F))).astype(F))
    return (((g * sig).astype(F)) * u).astype(F)


GELU_A = F(-2.0 * np.sqrt(2.0 / np.pi))                  # `compiler/frontend/hf_generic.py:848-849`
GELU_B = F(-2.0 * np.sqrt(2.0 / np.pi) * 0.044715)


def gelu_gate(g, u):
    """h = (g*RECIP(EXP(z) + 1))*u, z = g*(A + (g*g)*B): GELU's tanh approximation
    with multiplies, adds, EXP and RECIP only (`compiler/frontend/hf_generic.py:840-856`
    SaGELUTanh; the gated MLP's act(gate) * up)."""
    g = np.asarray(g, F)
    with np.errstate(over="ignore", invalid="ignore"):                  # (inf, NaN: as the device)
        z = (g * (GELU_A + ((g * g).astype(F) * GELU_B).astype(F)).astype(F)).astype(F)
        sig = sfu_recip((sfu_exp(z) + F(1)).astype(F))
        return (((g * sig).astype(F)) * u).astype(F)


def gate(g, u, act="silu"):
    return gelu_gate(g, u) if act == "gelu_tanh" else silu_gate(g, u)


def quantize_rows(wt):
    """Offline per-output-channel int8 (`llm/ref_model.py:142-148`;
    `hf_generic._quantize_rows` :558-565 sets s = 1 for all-zero rows):
    s = amax/127, q = i8(w/s)."""
    wt = np.asarray(wt, F)
    s = (np.abs(wt).max(axis=-1) / F(127)).astype(F)
    s = np.where(s == 0, F(1), s).astype(F)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = to_i8(wt / s[..., None])
    return q, s
