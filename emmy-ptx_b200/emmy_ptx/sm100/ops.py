"""Elementwise operators as sm_100a PTX instruction sequences.

The operator *semantics* are the contract with the reference: for every op
name the reference lowers (emmy_ptx/compiler.py:1047-1404) this table emits
an instruction sequence that computes the same function -- the same
``*.approx`` hardware approximations where the reference uses them (ex2 for
exp/sigmoid/tanh, rsqrt.approx, lg2.approx), IEEE ``.rn`` division, square
root and reciprocal, truncating ``div.s32``/``rem.s32`` for integer
``floor_divide``/``remainder`` (compiler.py:1383-1385) -- so results agree to
the ulp, and integers bit for bit.  ``int_semantics="torch"`` switches the
two integer ops to floor division / divisor-signed remainder (torch's
meaning), which the reference does not implement.

The table is organised by (op, dtype class) -> emitter and keeps the
operand-promotion rules of the reference (compiler.py:1035-1045, 1114-1119,
1311-1319).
"""

from __future__ import annotations

from .ptx import KernelBuilder, f32_hex, f64_hex

F32_ONLY = frozenset({
    "exp", "exp_fast", "sign", "log", "log2", "log10", "softplus",
    "sin", "cos", "tan", "pow", "relu", "sigmoid", "silu", "tanh",
    "erf", "gelu", "gelu_tanh", "reciprocal", "sqrt", "rsqrt", "fma",
})

_ALIASES = {"float": "f32", "double": "f64", "half": "f16", "int": "s32",
            "bool": "s32", "i32": "s32", "i64": "s64", "u32": "s32"}

LOG2E = 1.4426950408889634


class LoweringError(Exception):
    pass


def dtype_name(dt) -> str:
    if dt is None:
        return None
    name = getattr(dt, "name", str(dt))
    return _ALIASES.get(name, name)


def is_float(dt) -> bool:
    n = dtype_name(dt)
    return n.startswith("f") or n == "bf16"


def promoted(dts) -> str:
    if "f64" in dts:
        return "f64"
    if "f32" in dts:
        return "f32"
    return "s32"


class Ops:
    """Emits elementwise operations into a KernelBuilder.

    Values are ``(register, dtype)`` pairs.  Constants are cached per
    builder, and a ``remainder`` whose quotient was already computed reuses
    it (``r = a - q*b``), which is exact.
    """

    def __init__(self, b: KernelBuilder, int_semantics: str = "reference"):
        if int_semantics not in ("reference", "torch"):
            raise ValueError("int_semantics must be 'reference' or 'torch'")
        self.b = b
        self.int_semantics = int_semantics
        self._consts: dict = {}
        self._quot: dict = {}

    # -- constants and conversions ------------------------------------------
    def const(self, value, dt):
        dt = dtype_name(dt)
        key = (dt, repr(value))
        if key in self._consts:
            return self._consts[key]
        b = self.b
        r = b.reg_for(dt)
        if dt == "f32":
            b.ins(f"mov.f32 {r}, {f32_hex(value)};")
        elif dt == "f64":
            b.ins(f"mov.f64 {r}, {f64_hex(value)};")
        elif dt == "pred":
            b.ins(f"setp.ne.u32 {r}, {1 if value else 0}, 0;")
        else:
            b.ins(f"mov.s32 {r}, {int(value)};")
        self._consts[key] = (r, dt)
        return r, dt

    def coerce(self, v, target):
        """compiler.py:669-722 conversion rules."""
        reg, dt = v
        target = dtype_name(target)
        b = self.b
        if dt == "pred":
            t = b.reg("r")
            b.ins(f"selp.b32 {t}, 1, 0, {reg};")
            reg, dt = t, "s32"
        if dt == target:
            return reg
        if dt in ("u8", "s32", "u32") and target in ("u8", "s32", "u32"):
            return reg                      # the same 32-bit register (u8 zero-extended)
        # 16-bit floats: exact widening to f32; narrowing rounds to nearest
        # even; other types go through f32
        if dt in ("f16", "bf16"):
            wide = b.reg("f")
            b.ins(f"cvt.f32.{dt} {wide}, {reg};")
            return self.coerce((wide, "f32"), target)
        if target in ("f16", "bf16"):
            f = self.coerce((reg, dt), "f32")
            out = b.reg("h")
            b.ins(f"cvt.rn.{target}.f32 {out}, {f};")
            return out
        if target in ("s32", "u32") and dt in ("s64", "u64"):
            out = b.reg("r")
            b.ins(f"cvt.s32.s64 {out}, {reg};")
            return out
        if target in ("s64", "u64") and dt in ("s32", "u32"):
            out = b.reg("rd")
            b.ins(f"cvt.s64.s32 {out}, {reg};")
            return out
        if is_float(target) and not is_float(dt):
            out = b.reg_for(target)
            src = "s64" if dt in ("s64", "u64") else "s32"
            b.ins(f"cvt.rn.{target}.{src} {out}, {reg};")
            return out
        if not is_float(target) and is_float(dt):
            out = b.reg("r")
            b.ins(f"cvt.rzi.s32.{dt} {out}, {reg};")
            return out
        out = b.reg_for(target)
        if dt == "f32" and target == "f64":
            b.ins(f"cvt.f64.f32 {out}, {reg};")
        else:
            b.ins(f"cvt.rn.f32.f64 {out}, {reg};")
        return out

    # -- helpers -----------------------------------------------------------
    def _f(self, fmt, *regs, kind="f"):
        out = self.b.reg(kind)
        self.b.ins(fmt.format(out, *regs))
        return out

    def _ex2(self, t):
        return self._f("ex2.approx.f32 {0}, {1};", t)

    def _exp(self, x):
        t = self._f("mul.f32 {0}, {1}, " + f32_hex(LOG2E) + ";", x)
        return self._ex2(t)

    def _rcp(self, x):
        return self._f("rcp.rn.f32 {0}, {1};", x)

    def _tanh(self, x):
        b = self.b
        ax = self._f("abs.f32 {0}, {1};", x)
        y = self._f("mul.f32 {0}, {1}, " + f32_hex(-2.8853900817779268) + ";", ax)
        e = self._ex2(y)
        num = self._f("sub.f32 {0}, 0f3F800000, {1};", e)
        den = self._f("add.f32 {0}, {1}, 0f3F800000;", e)
        ratio = self._f("div.rn.f32 {0}, {1}, {2};", num, den)
        p = b.reg("p")
        b.ins(f"setp.lt.f32 {p}, {x}, 0f00000000;")
        neg = self._f("neg.f32 {0}, {1};", ratio)
        return self._f("selp.f32 {0}, {1}, {2}, " + p + ";", neg, ratio)

    def _erf(self, t):
        # Abramowitz & Stegun 7.1.26, the polynomial the reference uses
        b = self.b
        a = self._f("abs.f32 {0}, {1};", t)
        nsq = self._f("mul.f32 {0}, {1}, {1};", a)
        nsq = self._f("neg.f32 {0}, {1};", nsq)
        ex = self._exp(nsq)
        tau = self._f("fma.rn.f32 {0}, {1}, " + f32_hex(0.3275911) + ", 0f3F800000;", a)
        iv = self._rcp(tau)
        h = self._f("fma.rn.f32 {0}, " + f32_hex(1.061405429) + ", {1}, " + f32_hex(-1.453152027) + ";", iv)
        for c in (1.421413741, -0.284496736, 0.254829592):
            h = self._f("fma.rn.f32 {0}, {1}, {2}, " + f32_hex(c) + ";", h, iv)
        h = self._f("mul.f32 {0}, {1}, {2};", h, iv)
        tail = self._f("mul.f32 {0}, {1}, {2};", h, ex)
        pos = self._f("sub.f32 {0}, 0f3F800000, {1};", tail)
        p = b.reg("p")
        b.ins(f"setp.lt.f32 {p}, {t}, 0f00000000;")
        neg = self._f("neg.f32 {0}, {1};", pos)
        return self._f("selp.f32 {0}, {1}, {2}, " + p + ";", neg, pos)

    def _pow(self, x, y):
        b = self.b
        ax = self._f("abs.f32 {0}, {1};", x)
        l2 = self._f("lg2.approx.f32 {0}, {1};", ax)
        pr = self._f("mul.f32 {0}, {1}, {2};", l2, y)
        mag = self._ex2(pr)
        yi = self._f("cvt.rmi.f32.f32 {0}, {1};", y)
        p_int = b.reg("p")
        b.ins(f"setp.eq.f32 {p_int}, {y}, {yi};")
        half = self._f("mul.f32 {0}, {1}, 0f3F000000;", y)
        qh = self._f("cvt.rmi.f32.f32 {0}, {1};", half)
        t = self._f("fma.rn.f32 {0}, {1}, 0fC0000000, {2};", qh, y)
        p_odd, p_neg, p_sn, p_nan, p_00 = b.regs("p", 5)
        b.ins(f"setp.eq.f32 {p_odd}, {t}, 0f3F800000;")
        b.ins(f"setp.lt.f32 {p_neg}, {x}, 0f00000000;")
        b.ins(f"and.pred {p_sn}, {p_neg}, {p_int};")
        b.ins(f"and.pred {p_sn}, {p_sn}, {p_odd};")
        neg = self._f("neg.f32 {0}, {1};", mag)
        signed = self._f("selp.f32 {0}, {1}, {2}, " + p_sn + ";", neg, mag)
        b.ins(f"and.pred {p_nan}, {p_neg}, !{p_int};")
        out = self._f("selp.f32 {0}, 0f7FC00000, {1}, " + p_nan + ";", signed)
        p_az, p_yz = b.regs("p", 2)
        b.ins(f"setp.eq.f32 {p_az}, {ax}, 0f00000000;")
        b.ins(f"setp.eq.f32 {p_yz}, {y}, 0f00000000;")
        b.ins(f"and.pred {p_00}, {p_az}, {p_yz};")
        return self._f("selp.f32 {0}, 0f3F800000, {1}, " + p_00 + ";", out)

    # -- integer division ------------------------------------------------------
    def _idiv(self, a, bb, floor=False):
        """Quotient of a / bb: truncating (``div.s32``, the reference's
        lowering), or floored for ``floor_divide``/``remainder`` under
        ``int_semantics="torch"``."""
        floor = floor and self.int_semantics == "torch"
        key = (a, bb, floor)
        if key in self._quot:
            return self._quot[key]
        q = self.b.reg("r")
        self.b.ins(f"div.s32 {q}, {a}, {bb};")
        if floor:
            # floor: subtract one when the remainder is nonzero and has the
            # opposite sign of the divisor
            prod, r, x = self.b.regs("r", 3)
            p1, p2 = self.b.regs("p", 2)
            self.b.ins(f"mul.lo.s32 {prod}, {q}, {bb};")
            self.b.ins(f"sub.s32 {r}, {a}, {prod};")
            self.b.ins(f"xor.b32 {x}, {r}, {bb};")
            self.b.ins(f"setp.ne.s32 {p1}, {r}, 0;")
            self.b.ins(f"setp.lt.s32 {p2}, {x}, 0;")
            self.b.ins(f"and.pred {p1}, {p1}, {p2};")
            q2 = self.b.reg("r")
            self.b.ins(f"selp.s32 {x}, 1, 0, {p1};")
            self.b.ins(f"sub.s32 {q2}, {q}, {x};")
            q = q2
        self._quot[key] = q
        return q

    def _irem(self, a, bb):
        q = self._idiv(a, bb, floor=True)
        prod = self.b.reg("r")
        self.b.ins(f"mul.lo.s32 {prod}, {q}, {bb};")
        r = self.b.reg("r")
        self.b.ins(f"sub.s32 {r}, {a}, {prod};")
        return r

    # -- dispatch --------------------------------------------------------------
    _CMP = {"greater": "gt", "greater_equal": "ge", "less": "lt", "less_equal": "le",
            "equal": "eq", "not_equal": "ne"}
    _FBIN = {"add": "add", "sum": "add", "subtract": "sub", "sub": "sub",
             "multiply": "mul", "prod": "mul", "divide": "div.rn", "true_divide": "div.rn",
             "maximum": "max", "minimum": "min", "max": "max", "min": "min",
             "amax": "max", "amin": "min"}
    _IBIN = {"add": "add.s32", "sum": "add.s32", "subtract": "sub.s32", "sub": "sub.s32",
             "multiply": "mul.lo.s32", "prod": "mul.lo.s32", "maximum": "max.s32",
             "minimum": "min.s32", "max": "max.s32", "min": "min.s32", "amax": "max.s32",
             "amin": "min.s32", "and": "and.b32", "or": "or.b32", "xor": "xor.b32",
             "left_shift": "shl.b32", "right_shift": "shr.s32",
             "bitwise_right_shift": "shr.s32"}

    def emit(self, op, args, dtype="f32"):
        """Emit op ``op`` over ``args`` (``[(reg, dtype)]``); statement dtype
        ``dtype``.  Returns ``(reg, dtype)``."""
        name = getattr(op, "name", str(op))
        dt = dtype_name(dtype) or "f32"
        b = self.b
        dts = [d for _, d in args]
        if name in self._CMP:
            tgt = promoted(dts)
            a0 = self.coerce(args[0], tgt)
            a1 = self.coerce(args[1], tgt)
            p = b.reg("p")
            b.ins(f"setp.{self._CMP[name]}.{tgt} {p}, {a0}, {a1};")
            return p, "pred"
        if name == "where":
            c, cdt = args[0]
            if cdt != "pred":
                p = b.reg("p")
                kind = "f32" if is_float(cdt) else "s32"
                zero = "0f00000000" if kind == "f32" else "0"
                b.ins(f"setp.ne.{kind} {p}, {c}, {zero};")
                c = p
            x = self.coerce(args[1], dt)
            y = self.coerce(args[2], dt)
            out = b.reg_for(dt)
            t = {"f32": "f32", "f64": "f64"}.get(dt, "b32")
            b.ins(f"selp.{t} {out}, {x}, {y}, {c};")
            return out, dt
        if name in ("negative", "neg"):
            reg, adt = args[0]
            out = b.reg_for(adt)
            b.ins(f"neg.{adt} {out}, {reg};")
            return out, adt
        if name in ("logical_and", "logical_or", "logical_not"):
            if name == "logical_not":
                reg, adt = args[0]
                p = b.reg("p")
                if adt == "pred":
                    b.ins(f"not.pred {p}, {reg};")
                else:
                    zero = {"f32": "0f00000000", "f64": "0d0000000000000000"}.get(adt, "0")
                    b.ins(f"setp.eq.{adt} {p}, {reg}, {zero};")
                return p, "pred"
            opc = name.split("_")[1]
            if dts == ["pred", "pred"]:
                p = b.reg("p")
                b.ins(f"{opc}.pred {p}, {args[0][0]}, {args[1][0]};")
                return p, "pred"
            x = self.coerce(args[0], "s32")
            y = self.coerce(args[1], "s32")
            out = b.reg("r")
            b.ins(f"{opc}.b32 {out}, {x}, {y};")
            return out, "s32"
        if name in F32_ONLY:
            regs = [self.coerce(a, "f32") for a in args]
            return self._f32_only(name, regs), "f32"
        if name in ("absolute", "abs"):
            if dt in ("f32", "f64"):
                x = self.coerce(args[0], dt)
                out = b.reg_for(dt)
                b.ins(f"abs.{dt} {out}, {x};")
                return out, dt
            if dt == "f16":
                raise LoweringError("unsupported float op abs for f16")
            x = self.coerce(args[0], "s32")
            out = b.reg("r")
            b.ins(f"abs.s32 {out}, {x};")
            return out, "s32"
        if name in ("copy", "pad"):
            x = self.coerce(args[0], dt)
            out = b.reg_for(dt)
            t = {"f32": "f32", "f64": "f64", "pred": "pred"}.get(dt, "b32")
            b.ins(f"mov.{t} {out}, {x};")
            return out, dt
        if name == "bitcast":
            reg, src = args[0]
            if src == dt:
                return reg, dt
            kinds = {("f32", "s32"): ("r", "b32"), ("s32", "f32"): ("f", "b32"),
                     ("f64", "s64"): ("rd", "b64"), ("s64", "f64"): ("fd", "b64")}
            if (src, dt) not in kinds:
                raise LoweringError(f"unsupported bitcast {src} -> {dt}")
            kind, t = kinds[(src, dt)]
            out = b.reg(kind)
            b.ins(f"mov.{t} {out}, {reg};")
            return out, dt
        if name in ("from_f8e4m3", "from_f8e5m2"):
            return self._fp8_decode(name, args[0]), "f32"
        if is_float(dt):
            if dt == "f16":
                raise LoweringError(f"unsupported float op {name!r} for f16")
            regs = [self.coerce(a, dt) for a in args]
            if name in ("floor_divide", "remainder", "mod"):
                q = self._f(f"div.rn.{dt} {{0}}, {{1}}, {{2}};", regs[0], regs[1],
                            kind="f" if dt == "f32" else "fd")
                fl = self._f(f"cvt.rmi.{dt}.{dt} {{0}}, {{1}};", q,
                             kind="f" if dt == "f32" else "fd")
                if name == "floor_divide":
                    return fl, dt
                pr = self._f(f"mul.{dt} {{0}}, {{1}}, {{2}};", fl, regs[1],
                             kind="f" if dt == "f32" else "fd")
                return self._f(f"sub.{dt} {{0}}, {{1}}, {{2}};", regs[0], pr,
                               kind="f" if dt == "f32" else "fd"), dt
            base = self._FBIN.get(name)
            if base is None:
                raise LoweringError(f"unsupported float op {name!r}")
            out = b.reg_for(dt)
            b.ins(f"{base}.{dt} {out}, {regs[0]}, {regs[1]};")
            return out, dt
        regs = [self.coerce(a, "s32") for a in args]
        if name in ("divide", "true_divide", "floor_divide"):
            return self._idiv(regs[0], regs[1], floor=name == "floor_divide"), "s32"
        if name in ("remainder", "mod"):
            return self._irem(regs[0], regs[1]), "s32"
        ins = self._IBIN.get(name)
        if ins is None:
            raise LoweringError(f"unsupported integer op {name!r}")
        out = b.reg("r")
        b.ins(f"{ins} {out}, {regs[0]}, {regs[1]};")
        return out, "s32"

    def _fp8_decode(self, name, arg):
        """The low byte of ``arg`` as an fp8 code -> f32 (exact).  On sm_90
        and later the hardware converts a pair of codes to f16x2 (exact:
        both fp8 formats are contained in f16), then f16 -> f32; older
        targets assemble the f32 bit pattern from the code's fields."""
        b = self.b
        reg, dt = arg
        if dt not in ("s32", "u32", "u8", "b32"):
            reg = self.coerce(arg, "s32")
        hw = b.target in ("sm_90", "sm_90a", "sm_100", "sm_100a") and \
            tuple(int(x) for x in b.version.split(".")) >= (7, 8)
        if not hw:
            return self._fp8_decode_fields(name, reg)
        h = b.reg("h")
        b.ins(f"cvt.u16.u32 {h}, {reg};")
        b.ins(f"and.b16 {h}, {h}, 0x00FF;")
        pair = b.reg("r")
        fmt = "e4m3x2" if name == "from_f8e4m3" else "e5m2x2"
        b.ins(f"cvt.rn.f16x2.{fmt} {pair}, {h};")
        lo, hi = b.regs("h", 2)
        b.ins(f"mov.b32 {{{lo}, {hi}}}, {pair};")
        out = b.reg("f")
        b.ins(f"cvt.f32.f16 {out}, {lo};")
        return out

    def _fp8_decode_fields(self, name, code):
        """fp8 -> f32 from the code's sign / exponent / mantissa fields
        (OCP formats: E4M3 bias 7, S.1111.111 = NaN, no infinities; E5M2
        bias 15, exponent 31 = infinity (mantissa 0) or NaN)."""
        b = self.b
        E, M = (4, 3) if name == "from_f8e4m3" else (5, 2)
        bias = (1 << (E - 1)) - 1
        c, sgn, e, m, bits, sub = b.regs("r", 6)
        b.ins(f"and.b32 {c}, {code}, 255;")
        b.ins(f"shr.u32 {sgn}, {c}, 7;")
        b.ins(f"shl.b32 {sgn}, {sgn}, 31;")
        b.ins(f"bfe.u32 {e}, {c}, {M}, {E};")
        b.ins(f"and.b32 {m}, {c}, {(1 << M) - 1};")
        # normal: sign | (e - bias + 127) << 23 | m << (23 - M)
        b.ins(f"add.u32 {bits}, {e}, {127 - bias};")
        b.ins(f"shl.b32 {bits}, {bits}, 23;")
        b.ins(f"shl.b32 {sub}, {m}, {23 - M};")
        b.ins(f"or.b32 {bits}, {bits}, {sub};")
        b.ins(f"or.b32 {bits}, {bits}, {sgn};")
        out = b.reg("f")
        b.ins(f"mov.b32 {out}, {bits};")
        # subnormal (e == 0): m * 2^(1 - bias - M), signed
        fm, fs = b.regs("f", 2)
        b.ins(f"cvt.rn.f32.u32 {fm}, {m};")
        b.ins(f"mul.f32 {fm}, {fm}, {f32_hex(2.0 ** (1 - bias - M))};")
        b.ins(f"mov.b32 {sub}, {fm};")
        b.ins(f"or.b32 {sub}, {sub}, {sgn};")
        b.ins(f"mov.b32 {fs}, {sub};")
        pz = b.reg("p")
        b.ins(f"setp.eq.u32 {pz}, {e}, 0;")
        b.ins(f"selp.f32 {out}, {fs}, {out}, {pz};")
        ps, pn = b.regs("p", 2)
        emax = (1 << E) - 1
        if name == "from_f8e4m3":
            b.ins(f"setp.eq.u32 {ps}, {c}, 127;")
            b.ins(f"setp.eq.u32 {pn}, {c}, 255;")
            b.ins(f"or.pred {ps}, {ps}, {pn};")
            b.ins(f"selp.f32 {out}, 0f7FC00000, {out}, {ps};")
        else:
            inf = b.reg("r")
            b.ins(f"or.b32 {inf}, {sgn}, 0x7F800000;")
            fi = b.reg("f")
            b.ins(f"mov.b32 {fi}, {inf};")
            b.ins(f"setp.eq.u32 {ps}, {e}, {emax};")
            b.ins(f"setp.ne.u32 {pn}, {m}, 0;")
            b.ins(f"selp.f32 {fi}, 0f7FC00000, {fi}, {pn};")
            b.ins(f"selp.f32 {out}, {fi}, {out}, {ps};")
        return out

    def _f32_only(self, name, regs):
        x = regs[0]
        if name in ("exp", "exp_fast"):
            return self._exp(x)
        if name == "sign":
            p1, p2 = self.b.regs("p", 2)
            self.b.ins(f"setp.gt.f32 {p1}, {x}, 0f00000000;")
            self.b.ins(f"setp.lt.f32 {p2}, {x}, 0f00000000;")
            t = self._f("selp.f32 {0}, 0f3F800000, 0f00000000, " + p1 + ";")
            return self._f("selp.f32 {0}, 0fBF800000, {1}, " + p2 + ";", t)
        if name in ("log", "log2", "log10"):
            l2 = self._f("lg2.approx.f32 {0}, {1};", x)
            if name == "log2":
                return l2
            scale = 0.6931471805599453 if name == "log" else 0.3010299956639812
            return self._f("mul.f32 {0}, {1}, " + f32_hex(scale) + ";", l2)
        if name == "softplus":
            e = self._exp(x)
            s = self._f("add.f32 {0}, {1}, 0f3F800000;", e)
            l2 = self._f("lg2.approx.f32 {0}, {1};", s)
            return self._f("mul.f32 {0}, {1}, " + f32_hex(0.6931471805599453) + ";", l2)
        if name in ("sin", "cos"):
            return self._f(f"{name}.approx.f32 {{0}}, {{1}};", x)
        if name == "tan":
            s = self._f("sin.approx.f32 {0}, {1};", x)
            c = self._f("cos.approx.f32 {0}, {1};", x)
            return self._f("div.rn.f32 {0}, {1}, {2};", s, c)
        if name == "pow":
            return self._pow(x, regs[1])
        if name == "relu":
            return self._f("max.f32 {0}, {1}, 0f00000000;", x)
        if name in ("sigmoid", "silu"):
            t = self._f("mul.f32 {0}, {1}, " + f32_hex(-LOG2E) + ";", x)
            e = self._ex2(t)
            d = self._f("add.f32 {0}, {1}, 0f3F800000;", e)
            sig = self._rcp(d)
            if name == "sigmoid":
                return sig
            return self._f("mul.f32 {0}, {1}, {2};", x, sig)
        if name == "tanh":
            return self._tanh(x)
        if name == "erf":
            return self._erf(x)
        if name == "gelu":
            inner = self._f("mul.f32 {0}, {1}, " + f32_hex(0.7071067811865476) + ";", x)
            e = self._erf(inner)
            one = self._f("add.f32 {0}, {1}, 0f3F800000;", e)
            half = self._f("mul.f32 {0}, {1}, 0f3F000000;", one)
            return self._f("mul.f32 {0}, {1}, {2};", half, x)
        if name == "gelu_tanh":
            x2 = self._f("mul.f32 {0}, {1}, {1};", x)
            x3 = self._f("mul.f32 {0}, {1}, {2};", x2, x)
            inner = self._f("fma.rn.f32 {0}, {1}, " + f32_hex(0.044715) + ", {2};", x3, x)
            s = self._f("mul.f32 {0}, {1}, " + f32_hex(0.7978845608028654) + ";", inner)
            th = self._tanh(s)
            u = self._f("add.f32 {0}, {1}, 0f3F800000;", th)
            hx = self._f("mul.f32 {0}, {1}, 0f3F000000;", x)
            return self._f("mul.f32 {0}, {1}, {2};", hx, u)
        if name == "reciprocal":
            return self._rcp(x)
        if name == "sqrt":
            return self._f("sqrt.rn.f32 {0}, {1};", x)
        if name == "rsqrt":
            return self._f("rsqrt.approx.f32 {0}, {1};", x)
        if name == "fma":
            return self._f("fma.rn.f32 {0}, {1}, {2}, {3};", x, regs[1], regs[2])
        raise LoweringError(f"unsupported op {name!r}")
