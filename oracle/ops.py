"""Elementwise semantics of the reference's PTX lowering, restated in numpy.

TEST INFRASTRUCTURE (the CPU oracle).  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg may import this package; the product never
does.

Every function follows the instruction sequence the reference emits for the
op (file:line below are in emmy_ptx/compiler.py of the reference):

* values are numpy arrays over lanes, typed f32/f64/s32/pred;
* transcendental ``*.approx`` instructions (ex2, lg2, rsqrt, sin, cos) are
  evaluated in float64 and rounded once to f32 -- the hardware is within a
  few ulp of that, which the parity tolerances absorb;
* ``div.rn``/``rcp.rn``/``sqrt.rn``/``add``/``mul`` are IEEE f32 in numpy,
  as in PTX (ptxas may contract a mul+add into an fma; again ulp-level);
* integer division is C division (truncation toward zero) and remainder has
  the dividend's sign: ``div.s32``/``rem.s32`` (compiler.py:1383-1385,
  797-798), which is what the reference computes for ``floor_divide`` and
  ``remainder`` on int32 even though torch floors.
"""

from __future__ import annotations

import numpy as np

NP = {"f32": np.float32, "f64": np.float64, "s32": np.int32, "s64": np.int64,
      "pred": np.bool_, "f16": np.float16, "bf16": np.uint16,   # bf16: raw bits
      "u8": np.uint8}

_ALIASES = {"float": "f32", "double": "f64", "half": "f16", "int": "s32",
            "bool": "s32", "i32": "s32", "i64": "s64", "u32": "s32"}


def _fp8_table(exp_bits: int, man_bits: int, ieee_special: bool) -> np.ndarray:
    """f32 value of every fp8 code (sign, exponent, mantissa), from the OCP
    8-bit floating point formats: E4M3 (bias 7, no infinities, S.1111.111 is
    NaN, so the largest finite is 448) and E5M2 (bias 15, IEEE-style:
    exponent all ones is infinity / NaN)."""
    bias = (1 << (exp_bits - 1)) - 1
    out = np.zeros(256, np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        e = (code >> man_bits) & ((1 << exp_bits) - 1)
        m = code & ((1 << man_bits) - 1)
        emax = (1 << exp_bits) - 1
        if ieee_special and e == emax:
            v = sign * np.inf if m == 0 else np.nan
        elif not ieee_special and e == emax and m == (1 << man_bits) - 1:
            v = np.nan
        elif e == 0:
            v = sign * m * 2.0 ** (1 - bias - man_bits)
        else:
            v = sign * (1 + m / (1 << man_bits)) * 2.0 ** (e - bias)
        out[code] = v
    return out


F8E4M3 = _fp8_table(4, 3, False)
F8E5M2 = _fp8_table(5, 2, True)

# compiler.py:105-109
F32_ONLY_OPS = frozenset({
    "exp", "exp_fast", "sign", "log", "log2", "log10", "softplus",
    "sin", "cos", "tan", "pow", "relu", "sigmoid", "silu", "tanh",
    "erf", "gelu", "gelu_tanh", "reciprocal", "sqrt", "rsqrt", "fma",
})

LOG2E_F32 = np.float32(1.4426950408889634)       # 0f3FB8AA3B, compiler.py:1124


class OracleError(Exception):
    pass


def dtype_name(dt) -> str:
    """compiler.py:83-85."""
    if dt is None:
        return None
    name = getattr(dt, "name", str(dt))
    return _ALIASES.get(name, name)


def is_float(dt) -> bool:
    n = dtype_name(dt)
    return n.startswith("f") or n == "bf16"


def bf16_to_f32(bits):
    """bf16 bit patterns (uint16) -> f32, exactly."""
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    """f32 -> bf16 bits, round to nearest even (cvt.rn.bf16.f32); NaN stays
    a quiet NaN."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, np.float32))
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def promoted(dts) -> str:
    """compiler.py:1035-1045."""
    if "f64" in dts:
        return "f64"
    if "f32" in dts:
        return "f32"
    return "s32"


def as_type(v, dt):
    return np.asarray(v).astype(NP[dt], copy=False)


def _f64(x):
    return np.asarray(x, np.float64)


def cvt_rzi_s32(x):
    """cvt.rzi.s32.f32/f64: truncate toward zero, saturate, NaN -> 0."""
    x = _f64(x)
    with np.errstate(invalid="ignore"):
        y = np.trunc(np.nan_to_num(x, nan=0.0, posinf=2**31 - 1, neginf=-2**31))
    return np.clip(y, -2**31, 2**31 - 1).astype(np.int32)


def coerce(v, dt, target):
    """compiler.py:669-722: pred->s32 by selp 1/0, int->float cvt.rn,
    float->int cvt.rzi, f32<->f64 cvt."""
    dt = dtype_name(dt)
    target = dtype_name(target)
    if dt == "pred":
        v = np.where(v, np.int32(1), np.int32(0))
        dt = "s32"
    if dt == target:
        return v
    # 16-bit floats convert exactly to f32; everything else goes through f32
    # (f64 -> 16-bit rounds twice, as the lowering does)
    if dt == "f16":
        return coerce(np.asarray(v, np.float16).astype(np.float32), "f32", target)
    if dt == "bf16":
        return coerce(bf16_to_f32(v), "f32", target)
    if target == "f16":
        return np.asarray(coerce(v, dt, "f32"), np.float32).astype(np.float16)
    if target == "bf16":
        return f32_to_bf16(coerce(v, dt, "f32"))
    if target in ("s32", "s64") and not is_float(dt):
        return as_type(v, target)
    if is_float(target) and not is_float(dt):
        return as_type(v, target)
    if not is_float(target) and is_float(dt):
        return cvt_rzi_s32(v)
    if is_float(dt) and is_float(target):
        return as_type(v, target)
    return v


# ---- transcendental approximations ------------------------------------------
def ex2_approx(t):
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        return np.exp2(_f64(t)).astype(np.float32)


def lg2_approx(x):
    with np.errstate(divide="ignore", invalid="ignore"):
        return np.log2(_f64(x)).astype(np.float32)


def rsqrt_approx(x):
    with np.errstate(divide="ignore", invalid="ignore"):
        return (1.0 / np.sqrt(_f64(x))).astype(np.float32)


def rcp_rn(x):
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        return (np.float32(1.0) / np.asarray(x, np.float32)).astype(np.float32)


def fma_rn(a, b, c):
    return (_f64(a) * _f64(b) + _f64(c)).astype(np.float32)


def _c32(v):
    return np.float32(v)


def exp_f32(x):
    """compiler.py:1121-1127: ex2.approx(x * log2e)."""
    with np.errstate(over="ignore", invalid="ignore"):
        t = np.asarray(x, np.float32) * LOG2E_F32
    return ex2_approx(t)


def tanh_f32(x):
    """compiler.py:879-902."""
    x = np.asarray(x, np.float32)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        y = np.abs(x) * _c32(-2.8853900817779268)
        e = ex2_approx(y)
        ratio = (np.float32(1) - e) / (e + np.float32(1))
    return ratio * np.where(x < 0, np.float32(-1), np.float32(1))


def erf_f32(t):
    """compiler.py:904-944: Abramowitz & Stegun 7.1.26."""
    t = np.asarray(t, np.float32)
    a = np.abs(t)
    ex = exp_f32(-(a * a))
    tau = fma_rn(a, _c32(0.3275911), np.float32(1))
    iv = rcp_rn(tau)
    h = fma_rn(_c32(1.061405429), iv, _c32(-1.453152027))
    h = fma_rn(h, iv, _c32(1.421413741))
    h = fma_rn(h, iv, _c32(-0.284496736))
    h = fma_rn(h, iv, _c32(0.254829592))
    h5 = h * iv
    pos = np.float32(1) - h5 * ex
    return np.where(t < 0, -pos, pos).astype(np.float32)


def pow_f32(x, y):
    """compiler.py:946-1010."""
    x = np.asarray(x, np.float32)
    y = np.asarray(y, np.float32)
    ax = np.abs(x)
    with np.errstate(over="ignore", invalid="ignore"):
        mag = ex2_approx(lg2_approx(ax) * y)
    yi = np.floor(y)
    p_int = y == yi
    qh = np.floor(y * np.float32(0.5))
    p_odd = fma_rn(qh, np.float32(-2), y) == np.float32(1)
    p_neg = x < 0
    signed = np.where(p_neg & p_int & p_odd, -mag, mag)
    out = np.where(p_neg & ~p_int, np.float32(np.nan), signed)
    return np.where((ax == 0) & (y == 0), np.float32(1), out).astype(np.float32)


# ---- integer helpers ---------------------------------------------------------
def div_s32(a, b):
    """div.s32: C division, truncation toward zero (compiler.py:797, 1383)."""
    a = np.asarray(a, np.int64)
    b = np.asarray(b, np.int64)
    with np.errstate(divide="ignore", invalid="ignore"):
        bb = np.where(b == 0, 1, b)
        q = np.abs(a) // np.abs(bb)
        q = np.where((a < 0) != (bb < 0), -q, q)
    return np.where(b == 0, -1, q).astype(np.int64).astype(np.int32)


def floor_div_s32(a, b):
    """``floor_divide`` on int32 under the backend's ``int_semantics="torch"``:
    the truncating quotient, less one when the remainder is nonzero and its
    sign differs from the divisor's -- torch's floor division for b != 0.
    Restated from the fix-up the backend emits after ``div.s32`` (so b == 0
    gives what that sequence gives, with div.s32's -1 quotient)."""
    q = div_s32(a, b).astype(np.int64)
    r = _wrap32(np.asarray(a, np.int64) - _wrap32(q * np.asarray(b, np.int64)))
    fix = (r != 0) & ((r.astype(np.int64) ^ np.asarray(b, np.int64)) < 0)
    return _wrap32(q - fix.astype(np.int64))


def floor_rem_s32(a, b):
    """``remainder`` under ``int_semantics="torch"``: a - floor_div(a, b) * b,
    which has the divisor's sign (torch.remainder) for b != 0."""
    q = floor_div_s32(a, b).astype(np.int64)
    return _wrap32(np.asarray(a, np.int64) - _wrap32(q * np.asarray(b, np.int64)))


def rem_s32(a, b):
    """rem.s32: sign of the dividend (compiler.py:798, 1384)."""
    a64 = np.asarray(a, np.int64)
    b64 = np.asarray(b, np.int64)
    q = div_s32(a, b).astype(np.int64)
    r = a64 - q * np.where(b64 == 0, 0, b64)
    return np.where(b64 == 0, a64, r).astype(np.int32)


def _wrap32(x):
    return np.asarray(x, np.int64).astype(np.int32)


def shl_b32(a, b):
    """shl.b32: shift amounts above 32 clamp to 32 (all bits out)."""
    a = np.asarray(a, np.int64) & 0xFFFFFFFF
    s = np.clip(np.asarray(b, np.int64) & 0xFFFFFFFF, 0, 32)
    return _wrap32((a << s) & 0xFFFFFFFF)


def shr_s32(a, b):
    """shr.s32: arithmetic; amounts above 32 clamp (sign fill)."""
    a = np.asarray(a, np.int32).astype(np.int64)
    s = np.clip(np.asarray(b, np.int64) & 0xFFFFFFFF, 0, 31)
    return (a >> s).astype(np.int32)


def _int_arith(op, a, b):
    a64 = np.asarray(a, np.int64)
    b64 = np.asarray(b, np.int64)
    if op == "add":
        return _wrap32(a64 + b64)
    if op == "sub":
        return _wrap32(a64 - b64)
    if op == "mul":
        return _wrap32((a64 * b64) & 0xFFFFFFFF)
    if op == "div":
        return div_s32(a, b)
    if op == "rem":
        return rem_s32(a, b)
    if op == "max":
        return np.maximum(a64, b64).astype(np.int32)
    if op == "min":
        return np.minimum(a64, b64).astype(np.int32)
    if op == "and":
        return _wrap32(a64 & b64)
    if op == "or":
        return _wrap32(a64 | b64)
    if op == "xor":
        return _wrap32(a64 ^ b64)
    if op == "shl":
        return shl_b32(a, b)
    if op == "shr":
        return shr_s32(a, b)
    raise OracleError(f"unsupported integer op {op!r}")


def _float_arith(op, a, b, dt):
    t = NP[dt]
    a = np.asarray(a, t)
    b = np.asarray(b, t)
    with np.errstate(all="ignore"):
        if op == "add":
            return (a + b).astype(t)
        if op == "sub":
            return (a - b).astype(t)
        if op == "mul":
            return (a * b).astype(t)
        if op == "div":
            return (a / b).astype(t)
        if op == "max":            # max.f32: a NaN operand yields the other one
            return np.fmax(a, b).astype(t)
        if op == "min":
            return np.fmin(a, b).astype(t)
    raise OracleError(f"unsupported float binary op {op!r}")


# compiler.py:1334-1367 (float) and 1374-1398 (integer) op tables
_FLOAT_OPS = {
    "add": "add", "sum": "add", "subtract": "sub", "sub": "sub",
    "multiply": "mul", "prod": "mul", "divide": "div", "true_divide": "div",
    "maximum": "max", "minimum": "min", "max": "max", "min": "min",
    "amax": "max", "amin": "min",
}
_INT_OPS = {
    "add": "add", "sum": "add", "subtract": "sub", "sub": "sub",
    "multiply": "mul", "prod": "mul", "divide": "div", "true_divide": "div",
    "floor_divide": "div", "remainder": "rem", "mod": "rem",
    "maximum": "max", "minimum": "min", "max": "max", "min": "min",
    "amax": "max", "amin": "min", "and": "and", "or": "or", "xor": "xor",
    "left_shift": "shl", "right_shift": "shr", "bitwise_right_shift": "shr",
}
_CMP = {"greater": np.greater, "greater_equal": np.greater_equal,
        "less": np.less, "less_equal": np.less_equal, "equal": np.equal,
        "not_equal": np.not_equal}


def op_on_values(name, args, arg_dts, dtype="f32", int_semantics="reference"):
    """The value of elementwise op ``name`` (compiler.py:1047-1404).

    ``args`` are lane arrays with dtypes ``arg_dts``; ``dtype`` is the
    statement's dtype.  Returns ``(value, dtype)``.  ``int_semantics``
    "torch" gives int32 ``floor_divide``/``remainder`` torch's floored
    meaning, as the backend's option of that name does; the default is the
    reference's truncating ``div.s32``/``rem.s32``.
    """
    name = getattr(name, "name", str(name))
    dt = dtype_name(dtype) or "f32"
    arg_dts = [dtype_name(d) for d in arg_dts]

    if name in _CMP:                                       # 1054-1070
        target = promoted(arg_dts)
        a = coerce(args[0], arg_dts[0], target)
        b = coerce(args[1], arg_dts[1], target)
        return _CMP[name](a, b), "pred"
    if name == "where":                                    # 1072-1084
        cond = args[0] if arg_dts[0] == "pred" else (np.asarray(args[0]) != 0)
        a = coerce(args[1], arg_dts[1], dt)
        b = coerce(args[2], arg_dts[2], dt)
        return np.where(cond, a, b).astype(NP[dt]), dt
    if name in ("negative", "neg"):                        # 1086-1091
        adt = arg_dts[0]
        with np.errstate(over="ignore"):
            if is_float(adt):
                return (-np.asarray(args[0], NP[adt])).astype(NP[adt]), adt
            return _wrap32(-np.asarray(args[0], np.int64)), adt
    if name in ("logical_and", "logical_or", "logical_not"):   # 1093-1113
        if name == "logical_not":
            if arg_dts[0] == "pred":
                return ~np.asarray(args[0], bool), "pred"
            return np.asarray(args[0]) == 0, "pred"
        if arg_dts[0] == "pred" and arg_dts[1] == "pred":
            f = np.logical_and if name == "logical_and" else np.logical_or
            return f(args[0], args[1]), "pred"
        a = coerce(args[0], arg_dts[0], "s32")
        b = coerce(args[1], arg_dts[1], "s32")
        return _int_arith("and" if name == "logical_and" else "or", a, b), "s32"

    if name in F32_ONLY_OPS:                               # 1118-1119
        args = [coerce(a, d, "f32") for a, d in zip(args, arg_dts)]
        arg_dts = ["f32"] * len(args)

    if name in ("exp", "exp_fast"):                        # 1121-1127
        return exp_f32(args[0]), "f32"
    if name == "sign":                                     # 1129-1139
        x = args[0]
        return np.where(x > 0, np.float32(1), np.where(x < 0, np.float32(-1), np.float32(0))), "f32"
    if name in ("log", "log2", "log10"):                   # 1141-1148
        l2 = lg2_approx(args[0])
        if name == "log2":
            return l2, "f32"
        scale = 0.6931471805599453 if name == "log" else 0.3010299956639812
        return (l2 * _c32(scale)).astype(np.float32), "f32"
    if name == "softplus":                                 # 1150-1158
        with np.errstate(over="ignore"):
            s = exp_f32(args[0]) + np.float32(1)
        return (lg2_approx(s) * _c32(0.6931471805599453)).astype(np.float32), "f32"
    if name in ("sin", "cos", "tan"):                      # 1160-1172
        x = _f64(args[0])
        if name == "sin":
            return np.sin(x).astype(np.float32), "f32"
        if name == "cos":
            return np.cos(x).astype(np.float32), "f32"
        with np.errstate(divide="ignore", invalid="ignore"):
            return (np.sin(x).astype(np.float32) / np.cos(x).astype(np.float32)), "f32"
    if name == "pow":                                      # 1174-1176
        return pow_f32(args[0], args[1]), "f32"
    if name == "relu":                                     # 1178-1181
        return np.fmax(args[0], np.float32(0)).astype(np.float32), "f32"
    if name in ("sigmoid", "silu"):                        # 1183-1199
        x = np.asarray(args[0], np.float32)
        with np.errstate(over="ignore"):
            t = (-x) * LOG2E_F32
            sig = rcp_rn(ex2_approx(t) + np.float32(1))
        if name == "sigmoid":
            return sig, "f32"
        return (x * sig).astype(np.float32), "f32"
    if name == "tanh":                                     # 1201-1202
        return tanh_f32(args[0]), "f32"
    if name in ("erf", "gelu", "gelu_tanh"):               # 1204-1234
        x = np.asarray(args[0], np.float32)
        if name == "gelu_tanh":
            x3 = x * x * x
            inner = fma_rn(x3, _c32(0.044715), x)
            th = tanh_f32(inner * _c32(0.7978845608028654))
            return ((x * np.float32(0.5)) * (th + np.float32(1))).astype(np.float32), "f32"
        if name == "gelu":
            e = erf_f32(x * _c32(0.7071067811865476))
            return ((np.float32(0.5) * (e + np.float32(1))) * x).astype(np.float32), "f32"
        return erf_f32(x), "f32"
    if name == "reciprocal":                               # 1236-1239
        return rcp_rn(args[0]), "f32"
    if name in ("absolute", "abs"):                        # 1241-1254
        if dt == "f64":
            return np.abs(np.asarray(args[0], np.float64)), "f64"
        if is_float(dt):
            return np.abs(np.asarray(args[0], np.float32)), "f32"
        return _wrap32(np.abs(np.asarray(args[0], np.int64))), "s32"
    if name in ("copy", "pad"):                            # 1271-1274
        return coerce(args[0], arg_dts[0], dt), dt
    if name == "bitcast":                                  # 1276-1295
        src = arg_dts[0] if arg_dts else dt
        if src == dt:
            return np.asarray(args[0], NP[dt]), dt
        pair = {("f32", "s32"): np.int32, ("s32", "f32"): np.float32,
                ("f64", "s64"): np.int64, ("s64", "f64"): np.float64}.get((src, dt))
        if pair is None:
            raise OracleError(f"unsupported bitcast {src} -> {dt}")
        return np.ascontiguousarray(args[0], NP[src]).view(pair), dt
    if name in ("sqrt", "rsqrt"):                          # 1297-1301
        if name == "sqrt":
            with np.errstate(invalid="ignore"):
                return np.sqrt(np.asarray(args[0], np.float32)), "f32"
        return rsqrt_approx(args[0]), "f32"
    if name == "fma":                                      # 1303-1306
        return fma_rn(*args[:3]), "f32"
    if name in ("from_f8e4m3", "from_f8e5m2"):
        # the low byte of the operand is an fp8 code; the value is exact in f32
        table = F8E4M3 if name == "from_f8e4m3" else F8E5M2
        codes = np.asarray(args[0]).astype(np.int64) & 0xFF
        return table[codes], "f32"

    if is_float(dt):                                       # 1311-1372
        if dt == "f16":
            raise OracleError(f"unsupported float op {name!r} for f16")
        args = [coerce(a, d, dt) for a, d in zip(args, arg_dts)]
        if name in ("floor_divide", "remainder", "mod"):   # 1320-1333
            with np.errstate(all="ignore"):
                q = (args[0] / args[1]).astype(NP[dt])
                fl = np.floor(q)
                if name == "floor_divide":
                    return fl, dt
                return (args[0] - fl * args[1]).astype(NP[dt]), dt
        op = _FLOAT_OPS.get(name)
        if op is None:
            raise OracleError(f"unsupported float op {name!r}")
        return _float_arith(op, args[0], args[1], dt), dt

    op = _INT_OPS.get(name)                                # 1374-1404
    if op is None:
        raise OracleError(f"unsupported integer op {name!r}")
    args = [coerce(a, d, "s32") for a, d in zip(args, arg_dts)]
    if int_semantics == "torch" and name in ("floor_divide", "remainder", "mod"):
        f = floor_div_s32 if name == "floor_divide" else floor_rem_s32
        return f(args[0], args[1]), "s32"
    return _int_arith(op, args[0], args[1]), "s32"


def binary_expr(op, a, adt, b, bdt):
    """BinaryExpr in index/condition expressions (compiler.py:724-813)."""
    adt, bdt = dtype_name(adt), dtype_name(bdt)
    if op in ("==", "!=", "<", "<=", ">", ">="):
        target = "f64" if "f64" in (adt, bdt) else ("f32" if (is_float(adt) or is_float(bdt)) else "s32")
        a = coerce(a, adt, target)
        b = coerce(b, bdt, target)
        f = {"==": np.equal, "!=": np.not_equal, "<": np.less, "<=": np.less_equal,
             ">": np.greater, ">=": np.greater_equal}[op]
        return f(a, b), "pred"
    if op in ("and", "or"):
        if adt == "pred" and bdt == "pred":
            f = np.logical_and if op == "and" else np.logical_or
            return f(a, b), "pred"
        return _int_arith(op, a, b), "s32"
    target = "f64" if "f64" in (adt, bdt) else ("f32" if (is_float(adt) or is_float(bdt)) else "s32")
    a = coerce(a, adt, target)
    b = coerce(b, bdt, target)
    if target in ("f32", "f64"):
        fop = {"+": "add", "-": "sub", "*": "mul", "/": "div", "maximum": "max",
               "minimum": "min", "max": "max", "min": "min"}.get(op)
        if fop is None:
            raise OracleError(f"unsupported float binary op {op!r}")
        return _float_arith(fop, a, b, target), target
    iop = {"+": "add", "-": "sub", "*": "mul", "/": "div", "%": "rem", "and": "and",
           "or": "or", "xor": "xor", "maximum": "max", "minimum": "min", "max": "max",
           "min": "min", "<<": "shl", ">>": "shr"}.get(op)
    if iop is None:
        raise OracleError(f"unsupported integer binary op {op!r}")
    return _int_arith(iop, a, b), "s32"
