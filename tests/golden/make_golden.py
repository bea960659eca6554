"""Generate the golden vectors under tests/golden/ by running the REFERENCE's own Python functions.

Run it where the reference project is available, giving its checkout as the argument (or in
$NVFP4_REFERENCE_ROOT)::

    python tests/golden/make_golden.py <reference checkout>

The reference modules open a model checkpoint at import time, so they cannot be imported; instead the needed
function definitions are extracted with ``ast`` and executed in a fresh namespace:

* ``scripts/nvfp4_ref.py``   E2M1, e4m3_byte_to_val, E4M3, _pos_vals, quant_e4m3_pos, _fp4_mag, quant_fp4,
  unpack_fp4, pack_fp4, nvfp4_quant_rows (lines 33-82)
* ``scripts/ref_forward.py`` rmsnorm, gelu_tanh, softmax, router, experts (lines 67-83, 160-192), with the
  checkpoint readers ``load_f32`` / ``dequant_linear`` replaced by stubs that return synthetic tensors
* ``scripts/gen_fp4_gemm_testcase.py`` is executed as a script (its output directory is a temporary folder here)

Outputs (all small): quant_cases.npz, gemm_cases.npz, moe_case.npz.  The committed fixtures are what the tests
read; this script is only needed to regenerate them.
"""
from __future__ import annotations

import ast
import os
import pathlib
import shutil
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
_REF_ARG = next((a for a in sys.argv[1:] if not a.startswith("-")), None) or os.environ.get("NVFP4_REFERENCE_ROOT")
if not _REF_ARG:
    raise SystemExit("usage: make_golden.py <reference checkout>  (or set NVFP4_REFERENCE_ROOT)")
REF = pathlib.Path(_REF_ARG)
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
import nvfp4_oracle as orc  # noqa: E402  (only for seeded input generation helpers)


def extract(path: pathlib.Path, names: list[str], ns: dict) -> dict:
    """Execute only the top-level defs/assignments named in ``names`` from ``path`` inside ``ns``."""
    tree = ast.parse(path.read_text())
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            keep.append(node)
        elif isinstance(node, ast.Assign):
            tg = [t.id for t in node.targets if isinstance(t, ast.Name)]
            if any(t in names for t in tg):
                keep.append(node)
    mod = ast.Module(body=keep, type_ignores=[])
    exec(compile(mod, str(path), "exec"), ns)
    missing = [n for n in names if n not in ns]
    assert not missing, f"not found in {path}: {missing}"
    return ns


def ref_nvfp4() -> dict:
    ns = {"np": np}
    return extract(REF / "scripts/nvfp4_ref.py",
                   ["E2M1", "e4m3_byte_to_val", "E4M3", "_pos_vals", "quant_e4m3_pos", "_fp4_mag", "quant_fp4",
                    "unpack_fp4", "pack_fp4", "nvfp4_quant_rows"], ns)


# ------------------------------------------------------------------------------------------------------------
# Quantiser cases
# ------------------------------------------------------------------------------------------------------------

def quant_inputs() -> dict[str, tuple[np.ndarray, np.float32]]:
    """name -> (float64 input matrix holding bf16- or fp32-representable values, fp32 global scale)."""
    cases = {}
    # (1) cfg1-style bf16 N(0,1) with 0.1% x50 outliers; global scale from the tensor amax.
    bits = orc.synth_bf16((48, 2816), 1.0, seed=11, outlier_frac=0.001)
    x = orc.bf16_bits_to_f32(bits).astype(np.float64)
    cases["bf16_outliers"] = (x, orc.global_scale_from_amax(np.abs(x).max()))
    # (2) test_linear_real-style fp32 activation 0.5*N(0,1), M=128 (scripts/nvfp4_ref.py:20-21,99-100).
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((128, 512)) * 0.5).astype(np.float32).astype(np.float64)
    cases["fp32_linear"] = (x, orc.global_scale_from_amax(np.abs(x).max()))
    # (3) weight-like N(0, 0.02) bf16, ragged rows (not a multiple of 128), K not a multiple of 64.
    bits = orc.synth_bf16((131, 208), 0.02, seed=3)
    x = orc.bf16_bits_to_f32(bits).astype(np.float64)
    cases["bf16_weight_ragged"] = (x, orc.global_scale_from_amax(np.abs(x).max()))
    # (4) edge blocks: exact e2m1 ties, exact e4m3 ties, zeros, -0.0, tiny negatives, subnormal scales,
    #     saturation.  Built from exactly representable values so the ties are real ties.
    cases["edges"] = edge_case_matrix()
    return cases


def edge_case_matrix() -> tuple[np.ndarray, np.float32]:
    g = np.float32(1.0)          # global scale 1: stored scale = e4m3(amax / 6)
    rows = []
    mids = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    # block amax 6 -> scale 1 exactly, local 1: element values ARE the e2m1 inputs; put every midpoint and
    # its float32 neighbours in.
    for m in mids:
        lo = np.nextafter(np.float32(m), np.float32(0))
        hi = np.nextafter(np.float32(m), np.float32(10))
        row = [6.0, m, -m, lo, hi, -lo, -hi, 0.0, -0.0, 1e-30, -1e-30, 0.5, 1.0, 6.0, -6.0, 3.0]
        rows.append(row)
    # e4m3 ties: amax/6 exactly halfway between neighbouring e4m3 values (1.0 and 1.125 -> 1.0625).
    for a6 in [1.0625, 1.1875, 3.25, 0.001953125 * 1.5, 0.0009765625, 0.0009765625 * 1.0001, 440.0, 500.0]:
        amax = a6 * 6.0
        row = [amax] + [amax * f for f in np.linspace(-1, 1, 15)]
        rows.append(row)
    rows.append([0.0] * 16)                       # all-zero block -> scale byte 0x80
    rows.append([-0.0] * 16)                      # negative zeros -> codes 0
    rows.append([-1e-38] * 8 + [1e-38] * 8)       # underflowing scale, tiny signed values
    rows.append([1e4] + [7.0] * 15)               # saturating scale (gscale*amax/6 > 448)
    x = np.array(rows, dtype=np.float32).astype(np.float64)
    # pad to 2 blocks per row so K = 32
    x = np.concatenate([x, x[:, ::-1] * 0.37], axis=1).astype(np.float32).astype(np.float64)
    return x, g


def make_quant(ns: dict) -> None:
    out = {}
    for name, (x, g) in quant_inputs().items():
        packed, sfb, deq = ns["nvfp4_quant_rows"](x, float(g))
        assert np.array_equal(x.astype(np.float32).astype(np.float64), x)   # inputs are fp32-exact
        out[f"{name}__x"] = x.astype(np.float32)
        out[f"{name}__gscale"] = np.float32(g)
        out[f"{name}__packed"] = packed
        out[f"{name}__sf"] = sfb
        if name == "edges":
            out[f"{name}__deq"] = deq
    # e4m3 encoder sweep: every e4m3 value, every midpoint and their float64 neighbours
    grid = ns["_pos_vals"]
    mids = (grid[1:] + grid[:-1]) / 2
    probe = np.concatenate([grid, mids, np.nextafter(mids, 0), np.nextafter(mids, 1e9),
                            [0.0, 1e-300, 2.0 ** -10, 447.0, 448.0, 460.0, 1e6]])
    b, v = ns["quant_e4m3_pos"](probe)
    out["e4m3_probe__x"], out["e4m3_probe__byte"], out["e4m3_probe__val"] = probe, b, v
    # e2m1 encoder sweep
    mag = ns["_fp4_mag"]
    m2 = (mag[1:] + mag[:-1]) / 2
    p = np.concatenate([mag, m2, np.nextafter(m2, 0), np.nextafter(m2, 9), [7.0, 100.0, 1e-300]])
    p = np.concatenate([p, -p, [-0.0]])
    c, _ = ns["quant_fp4"](p)
    out["e2m1_probe__x"], out["e2m1_probe__code"] = p, c
    np.savez_compressed(HERE / "quant_cases.npz", **out)


# ------------------------------------------------------------------------------------------------------------
# GEMM cases: the reference's own synthetic generator, run as a script
# ------------------------------------------------------------------------------------------------------------

def make_gemm() -> None:
    out = {}
    tmp = HERE / "_gen_tmp"
    for tag, dims in [("default", []), ("ragged", ["130", "200", "192"])]:
        if tmp.exists():
            shutil.rmtree(tmp)
        tmp.mkdir()
        argv = sys.argv
        try:
            sys.argv = ["gen_fp4_gemm_testcase.py", str(tmp)] + dims
            src = (REF / "scripts/gen_fp4_gemm_testcase.py").read_text()
            exec(compile(src, "gen_fp4_gemm_testcase.py", "exec"), {"__name__": "__main__"})
        finally:
            sys.argv = argv
        m, n, k = [int(v) for v in (tmp / "dims.txt").read_text().split()[:3]]
        ag, bg = [np.float32(float(v)) for v in (tmp / "dims.txt").read_text().split()[3:5]]
        out[f"{tag}__dims"] = np.array([m, n, k])
        out[f"{tag}__ag"], out[f"{tag}__bg"] = ag, bg
        out[f"{tag}__a_packed"] = np.fromfile(tmp / "A_packed.bin", np.uint8).reshape(m, k // 2)
        out[f"{tag}__b_packed"] = np.fromfile(tmp / "B_packed.bin", np.uint8).reshape(n, k // 2)
        out[f"{tag}__a_sf"] = np.fromfile(tmp / "A_scales.bin", np.uint8).reshape(m, k // 16)
        out[f"{tag}__b_sf"] = np.fromfile(tmp / "B_scales.bin", np.uint8).reshape(n, k // 16)
        out[f"{tag}__y_ref"] = np.fromfile(tmp / "Y_ref.bin", np.float32).reshape(m, n)
    shutil.rmtree(tmp)
    np.savez_compressed(HERE / "gemm_cases.npz", **out)


# ------------------------------------------------------------------------------------------------------------
# MoE case: reference router + experts on synthetic NVFP4 weights
# ------------------------------------------------------------------------------------------------------------

def make_moe(nv: dict) -> None:
    H, E, I, S = 256, 16, 64, 12
    rng = np.random.default_rng(5)

    def q_weight(shape, seed):
        bits = orc.synth_bf16(shape, 0.02, seed=seed)
        w = orc.bf16_bits_to_f32(bits).astype(np.float64)
        g = orc.global_scale_from_amax(np.abs(w).max())
        packed, sfb, deq = nv["nvfp4_quant_rows"](w, float(g))
        return packed, sfb, g, deq.astype(np.float32)

    weights = {}
    arrays = {}
    for e in range(E):
        for kind, shape, seed in [("gate_proj", (I, H), 1000 + e), ("up_proj", (I, H), 2000 + e),
                                  ("down_proj", (H, I), 3000 + e)]:
            packed, sfb, g, deq = q_weight(shape, seed)
            weights[f"experts.{e}.{kind}"] = deq
            arrays[f"{kind}__{e}__packed"], arrays[f"{kind}__{e}__sf"], arrays[f"{kind}__{e}__g"] = packed, sfb, g
    proj = orc.bf16_bits_to_f32(orc.synth_bf16((E, H), 0.02, seed=77))
    scale = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    pes = (1.0 + 0.05 * rng.standard_normal(E)).astype(np.float32)
    resid = orc.bf16_bits_to_f32(orc.synth_bf16((S, H), 1.0, seed=78))
    xm = orc.bf16_bits_to_f32(orc.synth_bf16((S, H), 1.0, seed=79))

    def load_f32(name):
        if name.endswith(".scale"):
            return scale
        if name.endswith(".proj.weight"):
            return proj
        if name.endswith(".per_expert_scale"):
            return pes
        raise KeyError(name)

    def dequant_linear(prefix):
        return weights[prefix.split("layers.0.", 1)[1]]

    ns = {"np": np, "H": H, "EPS": 1e-6, "load_f32": load_f32, "dequant_linear": dequant_linear}
    extract(REF / "scripts/ref_forward.py", ["rmsnorm", "gelu_tanh", "softmax", "router", "experts"], ns)
    topw, topi = ns["router"](resid, 0)
    out = ns["experts"](xm, topw, topi, 0)
    np.savez_compressed(HERE / "moe_case.npz", H=H, E=E, I=I, S=S, proj=proj, scale=scale, pes=pes,
                        resid=resid, xm=xm, topw=topw, topi=topi, out=out, **arrays)


def main() -> None:
    assert REF.exists(), f"reference project not found at {REF}"
    nv = ref_nvfp4()
    make_quant(nv)
    make_gemm()
    make_moe(nv)
    for f in sorted(HERE.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size} bytes")


if __name__ == "__main__":
    main()
