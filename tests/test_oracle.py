"""The CPU oracle: pinned against the reference's GPU results and against
closed-form numpy semantics."""

import hashlib
import tempfile
from pathlib import Path

import numpy as np
import pytest

import cases
from oracle import ops as O
from oracle import simt
from oracle.ops import OracleError
from tolerances import check_close

VECTORS = Path(__file__).resolve().parent / "golden" / "vectors"
PROBLEMS = Path(__file__).resolve().parent / "golden" / "problems"


def _digest(inputs):
    h = hashlib.sha256()
    for k in sorted(inputs):
        h.update(k.encode())
        h.update(np.ascontiguousarray(inputs[k]).tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("tag", list(cases.PARITY))
def test_oracle_matches_reference_gpu_vectors(tag):
    """Golden vectors: the reference compiler's PTX run on a B200
    (make_ref_vectors.py).  Integers bit-exact, floats within tolerance."""
    gold = np.load(VECTORS / f"{tag}.npz")
    p = cases.problem(tag)
    inputs = p.make_inputs()
    assert str(gold["__inputs_sha256__"]) == _digest(inputs), "seeded inputs changed"
    ir_path = next((PROBLEMS / tag).glob("*.ir.json"))
    want = simt.run_package(ir_path, inputs)
    for o in p.outputs:
        ok, msg = check_close(p.category, o, want[o], gold[o], inputs)
        assert ok, msg


def _closed_form(p, inp):
    if p.category == "pointwise_f32":
        x, y = inp["x"].astype(np.float64), inp["y"]
        return {"out": x / (1 + np.exp(-x)) + y}
    if p.category == "pointwise_i32":
        a, b = inp["a"].astype(np.int64), inp["b"].astype(np.int64)
        q = np.trunc(a / b).astype(np.int64)
        return {"q": q, "r": a - q * b, "s": ((a << 3).astype(np.int32) >> 1)}
    if p.category == "rmsnorm":
        x, w = inp["x"].astype(np.float64), inp["w"]
        return {"out": x / np.sqrt((x * x).mean(1, keepdims=True) + 1e-6) * w}
    if p.category == "softmax":
        x = inp["x"].astype(np.float64)
        e = np.exp(x - x.max(1, keepdims=True))
        return {"out": e / e.sum(1, keepdims=True)}
    if p.category == "colreduce_f64":
        return {"colsum": inp["x"].sum(0), "colmax": inp["x"].max(0)}
    if p.category == "rowsum_i32":
        return {"out": inp["x"].astype(np.int64).sum(1)}
    if p.category == "matmul":
        return {"C": inp["A"].astype(np.float64) @ inp["B"]}
    if p.category == "attention":
        q, k, v = (inp[n].astype(np.float64) for n in "qkv")
        s = q @ k.transpose(0, 1, 3, 2) * p.params["scale"]
        S = s.shape[-1]
        if p.params["causal"]:
            s = np.where(np.tril(np.ones((S, S), bool)), s, -np.inf)
        pr = np.exp(s - s.max(-1, keepdims=True))
        pr /= pr.sum(-1, keepdims=True)
        return {"out": pr @ v}
    if p.category == "pointwise_zoo":
        from math import erf
        x, y = inp["x"].astype(np.float64), inp["y"].astype(np.float64)
        verf = np.vectorize(erf)
        out = {"u_exp": np.exp(x), "u_log": np.log(y), "u_log2": np.log2(y),
               "u_log10": np.log10(y), "u_sqrt": np.sqrt(y), "u_rsqrt": 1 / np.sqrt(y),
               "u_reciprocal": 1 / y, "u_tanh": np.tanh(x), "u_erf": verf(x),
               "u_gelu": 0.5 * x * (1 + verf(x / np.sqrt(2))),
               "u_gelu_tanh": 0.5 * x * (1 + np.tanh(np.sqrt(2 / np.pi) * (x + 0.044715 * x ** 3))),
               "u_sigmoid": 1 / (1 + np.exp(-x)), "u_silu": x / (1 + np.exp(-x)),
               "u_softplus": np.log1p(np.exp(x)), "u_relu": np.maximum(x, 0),
               "u_abs": np.abs(x), "u_neg": -x, "u_sign": np.sign(x), "u_sin": np.sin(x),
               "u_cos": np.cos(x), "b_pow": y ** x, "b_maximum": np.maximum(y, x),
               "b_minimum": np.minimum(y, x), "b_divide": y / x, "b_subtract": y - x,
               "c_where": np.where(x > y, x, y), "c_fma": x * y + x}
        x32, y32 = inp["x"], inp["y"]
        q = np.floor((y32 / x32).astype(np.float32))
        out["b_floor_divide"] = q
        out["b_remainder"] = (y32 - q * x32).astype(np.float32)
        return out
    if p.category == "pointwise_mixed":
        d, f, n = inp["d"], inp["f"], inp["n"]
        fd = f.astype(np.float64)
        q = np.floor(d / fd)
        nn = (n.astype(np.int64) * n).astype(np.int32)
        return {"o_mul": (d + fd) * d, "o_fdiv": q, "o_frem": d - q * fd,
                "o_imax": np.maximum(nn, n), "o_pred": (fd < d).astype(np.int32),
                "o_half": f + n.astype(np.float32)}
    if p.category == "bit_ops":
        x, e, n, s = inp["x"], inp["e"], inp["n"], inp["s"]
        n64, s64 = n.astype(np.int64), s.astype(np.int64)
        # shl.b32 / shr.s32 clamp the count at 32
        shl = ((n64 << np.minimum(s64, 32)) & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
        shr = (n64 >> np.minimum(s64, 32)).astype(np.int32)
        with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
            pw = np.power(x.astype(np.float64), e.astype(np.float64))
        return {"o_bits": x.view(np.int32), "o_float": n.view(np.float32), "o_pad": x,
                "o_pow": pw, "o_xor": n ^ s, "o_shl": shl, "o_shr": shr}
    if p.category == "rowsum_f64":
        return {"out": inp["x"].sum(1)}
    if p.category == "offset_copy":
        o, cols = p.params["offset"], p.tensor("out")["shape"][1]
        return {"out": 2 * inp["x"][:, o:o + cols]}
    raise AssertionError(p.category)


@pytest.mark.parametrize("tag", list(cases.PARITY))
def test_oracle_matches_closed_form(tag):
    """The IR packages compute what their category means (integer
    floor_divide/remainder with the reference's truncation)."""
    p = cases.problem(tag)
    inp = p.make_inputs()
    with tempfile.TemporaryDirectory() as td:
        got = simt.run_problem(p, inp, td)
    want = _closed_form(p, inp)
    for o in p.outputs:
        w = want[o]
        if np.asarray(got[o]).dtype.kind == "i":
            np.testing.assert_array_equal(got[o], w)
        else:
            ok, msg = check_close(p.category, o, got[o], w.astype(got[o].dtype), inp)
            assert ok, msg


def test_integer_division_truncates_like_div_s32():
    a = np.array([7, -7, 7, -7, 0, -1], np.int32)
    b = np.array([2, 2, -2, -2, 5, 3], np.int32)
    np.testing.assert_array_equal(O.div_s32(a, b), [3, -3, -3, 3, 0, 0])
    np.testing.assert_array_equal(O.rem_s32(a, b), [1, -1, 1, -1, 0, -1])


def test_shifts_clamp_like_ptx():
    a = np.array([1, -8, 5], np.int32)
    np.testing.assert_array_equal(O.shl_b32(a, np.array([3, 1, 40])), [8, -16, 0])
    np.testing.assert_array_equal(O.shr_s32(a, np.array([0, 2, 40])), [1, -2, 0])


def test_float_remainder_is_floor_based():
    v, dt = O.op_on_values("remainder", [np.float32([-7.5]), np.float32([2.0])], ["f32", "f32"], "f32")
    assert dt == "f32" and v[0] == np.float32(0.5)


def test_max_ignores_nan_like_max_f32():
    v, _ = O.op_on_values("max", [np.float32([np.nan, 1.0]), np.float32([2.0, np.nan])],
                          ["f32", "f32"], "f32")
    np.testing.assert_array_equal(v, [2.0, 1.0])


def test_out_of_bounds_access_is_reported():
    from emmy_ptx import workloads
    from emmy_ptx.ir import BinaryExpr, Literal, Tile
    p = workloads.pointwise_f32(rows=4, cols=16)
    tile = p.kernel.body[0]
    bad_axes = (tile.axes[0], type(tile.axes[1])(tile.axes[1].name, type(tile.axes[1].extent)(5)))
    p.kernel = type(p.kernel)(p.kernel.name, p.kernel.inputs, p.kernel.outputs,
                              (Tile(bad_axes, tile.body, block_threads=256),))
    with tempfile.TemporaryDirectory() as td:
        with pytest.raises(OracleError, match="out-of-bounds"):
            simt.run_problem(p, p.make_inputs(), td)
    assert BinaryExpr and Literal


TORCH_CPU_TAGS = [t for t, (name, _) in cases.PARITY.items()
                  if name in ("pointwise_f32", "pointwise_i32", "rmsnorm", "softmax",
                              "colreduce_f64", "rowsum_i32", "matmul", "attention")]


@pytest.mark.parametrize("tag", TORCH_CPU_TAGS)
def test_torch_cpu_baseline_matches_reference_gpu_vectors(tag):
    """The timed CPU baseline (torch CPU operators, oracle/torch_cpu.py)
    computes what the reference's PTX computed on the B200: integers bit for
    bit (truncating int32 division, as the reference lowers it), floats within
    the parity tolerances."""
    import torch
    from oracle import torch_cpu
    p = cases.problem(tag)
    if not p.params.get("causal", True):
        pytest.skip("the CPU baseline times the causal configuration")
    gold = np.load(VECTORS / f"{tag}.npz")
    inputs = p.make_inputs()
    got = torch_cpu.run(p.category, {k: torch.from_numpy(v) for k, v in inputs.items()},
                        p.params)
    for o in p.outputs:
        ok, msg = check_close(p.category, o, got[o].numpy(), gold[o], inputs)
        assert ok, msg


def test_torch_int_semantics_mode_is_torch_floor_division(tmp_path):
    """The oracle's ``int_semantics="torch"`` mode (the backend option of the
    same name) gives int32 floor_divide / remainder exactly torch's results,
    negative operands included, while the default stays truncating."""
    import torch
    rng = np.random.default_rng(11)
    a = rng.integers(-2**20, 2**20, 5000).astype(np.int32)
    b = (rng.integers(1, 1000, 5000) * rng.choice([-1, 1], 5000)).astype(np.int32)
    ta, tb = torch.from_numpy(a), torch.from_numpy(b)
    q, _ = O.op_on_values("floor_divide", [a, b], ["s32", "s32"], "s32", "torch")
    r, _ = O.op_on_values("remainder", [a, b], ["s32", "s32"], "s32", "torch")
    assert (q == torch.floor_divide(ta, tb).numpy()).all()
    assert (r == torch.remainder(ta, tb).numpy()).all()
    qt, _ = O.op_on_values("floor_divide", [a, b], ["s32", "s32"], "s32")
    assert (qt == torch.div(ta, tb, rounding_mode="trunc").numpy()).all()
    assert (qt != q).any()
    # the whole int32 package under the torch mode
    p = cases.problem("pointwise_i32_33x100")
    inputs = p.make_inputs()
    got = simt.run_package(p.write(tmp_path), inputs, int_semantics="torch")
    ta, tb = torch.from_numpy(inputs["a"]), torch.from_numpy(inputs["b"])
    assert (got["q"].reshape(ta.shape) == torch.floor_divide(ta, tb).numpy()).all()
    assert (got["r"].reshape(ta.shape) == torch.remainder(ta, tb).numpy()).all()
