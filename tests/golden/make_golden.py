"""Generate golden vectors by running the reference implementation itself.

Run in a checkout that has the reference tree (not on the GPU box):

    python tests/golden/make_golden.py --reference /path/to/llima

It imports ``sima_lmm.gguf.gguf_conversion`` from the reference (with a stub for the
unused ``llama_cpp`` import, ``gguf_conversion.py:7``), feeds seeded synthetic GGUF
bytes through the reference's own ``unpack_gguf_tensor`` (``gguf_conversion.py:102-176``),
gguf-py's ``dequantize`` (the force_float path, ``:171-172``) and
``GgufModel._permute_qk_proj`` (``:314-332``), and writes one ``.npz`` per case into
this directory.  The requantization warning the reference logs
(``ggml_quant.py:879-880``) is captured as text.  Library versions are recorded in
``versions.json``.
"""
from __future__ import annotations

import argparse
import json
import logging
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from llima_b200.formats import FORMATS          # noqa: E402
from llima_b200.synth import gen_tensor_bytes   # noqa: E402


class _Capture(logging.Handler):
    def __init__(self):
        super().__init__(logging.WARNING)
        self.messages: list[str] = []

    def emit(self, record):
        self.messages.append(record.getMessage())


def _edge_kquant(fmt: str, n_sb: int, seed: int) -> np.ndarray:
    """K-quant super-blocks that hit the corner cases of the requantization:
    zero scales, zero mins, both zero, d = 0, dmin = 0, negative and subnormal f16
    constants, extreme ratios that clip, and all-equal codes."""
    f = FORMATS[fmt]
    rng = np.random.default_rng(seed)
    u = gen_tensor_bytes(fmt, n_sb * 256, seed).reshape(n_sb, f.unit_bytes).copy()
    if fmt == "Q6_K":
        # int8 sub-scales over the whole range, zero and negative d, subnormal d
        u[:, 192:208] = rng.integers(-128, 128, size=(n_sb, 16), dtype=np.int8).view(np.uint8)
        d = u[:, 208:210].copy().view(np.float16)
        d[0::7] = 0
        d[1::7] = -d[1::7]
        d[2::7] = np.float16(3e-7)          # subnormal f16
        d[3::7] = np.float16(60000.0)       # products overflow f16 -> inf
        u[:, 208:210] = d.view(np.uint8)
        return u.reshape(-1)
    d = u[:, 0:2].copy().view(np.float16)
    dmin = u[:, 2:4].copy().view(np.float16)
    sc_bytes = u[:, 4:16]
    for i in range(n_sb):
        case = i % 12
        if case == 0:
            sc_bytes[i] = 0                      # all scales and mins zero
        elif case == 1:
            d[i] = 0                             # S = 0 -> alternative scale
        elif case == 2:
            dmin[i] = 0                          # M = 0 (negated: -0.0)
        elif case == 3:
            d[i] = np.float16(1e-7)              # tiny S, large |r| -> sf < 1
            dmin[i] = np.float16(0.5)
        elif case == 4:
            d[i] = -d[i]                         # negative scale
        elif case == 5:
            dmin[i] = -dmin[i]                   # negative min (positive M)
        elif case == 6:
            d[i] = np.float16(6e-8)              # smallest subnormal
        elif case == 7:
            dmin[i] = np.float16(65504.0)        # M overflows f16 -> -inf
        elif case == 8:
            u[i, 16:] = 0xFF                     # all codes at the top
        elif case == 9:
            u[i, 16:] = 0x00                     # all codes zero
        elif case == 10:
            d[i] = np.float16(1e-4)
            dmin[i] = np.float16(1e-4)
            sc_bytes[i] = 0x41                   # equal small scales and mins
    u[:, 0:2] = d.view(np.uint8)
    u[:, 2:4] = dmin.view(np.uint8)
    return u.reshape(-1)


def _nonfinite(fmt: str, n_units: int, seed: int) -> np.ndarray:
    """Fully uniform random bytes: f16 constants include NaN, inf and huge values."""
    f = FORMATS[fmt]
    rng = np.random.default_rng(seed)
    return np.frombuffer(rng.bytes(n_units * f.unit_bytes), dtype=np.uint8).copy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout (the directory holding sima_lmm/)")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", choices=["all", "partition", "ggml_quant"], default="all",
                    help="partition: rewrite only partition.json; ggml_quant: only ggml_quant/*.npz")
    args = ap.parse_args()

    sys.path.insert(0, args.reference)
    sys.modules.setdefault("llama_cpp", types.SimpleNamespace(Llama=object))
    import gguf
    import ml_dtypes
    from gguf import GGMLQuantizationType as T
    from gguf import dequantize as gguf_dequantize
    from sima_lmm.gguf import gguf_conversion as gc

    cap = _Capture()
    logging.getLogger("sima_lmm.gguf.ggml_quant").addHandler(cap)
    out = Path(args.out)
    manifest = []
    if args.only == "ggml_quant":
        from sima_lmm.gguf import ggml_quant as gq
        write_ggml_quant(gq, cap, out / "ggml_quant", ml_dtypes, gguf)
        return

    def run(case: str, fmt: str, raw: np.ndarray, rows: int, cols: int, heads: int = 0):
        f = FORMATS[fmt]
        n_units = rows * cols // f.unit_values
        assert raw.size == n_units * f.unit_bytes
        data = raw.reshape(rows, -1) if fmt not in ("F32",) else raw.view(np.float32).reshape(rows, cols)
        tensor = types.SimpleNamespace(tensor_type=getattr(T, fmt), data=data,
                                       shape=np.array([cols, rows], dtype=np.uint64))
        cap.messages.clear()
        with np.errstate(all="ignore"):
            scales, codes = gc.unpack_gguf_tensor(tensor, False)
        warning = "\n".join(cap.messages)
        with np.errstate(all="ignore"):
            f32 = np.asarray(gguf_dequantize(data, getattr(T, fmt)), dtype=np.float32).reshape(rows, cols)
        rec = {"raw": raw, "rows": rows, "cols": cols, "fmt": fmt,
               "codes": codes.view(np.uint8) if codes.dtype == ml_dtypes.int4 else codes,
               "codes_dtype": str(codes.dtype), "f32": f32, "warning": warning}
        if scales is not None:
            rec["scales"] = scales
        if heads:
            ps, pw = gc.GgufModel._permute_qk_proj(None, scales, codes, heads)
            rec["perm_heads"] = heads
            rec["perm_codes"] = pw.view(np.uint8) if pw.dtype == ml_dtypes.int4 else pw
            if ps is not None:
                rec["perm_scales"] = ps
        np.savez_compressed(out / f"{case}.npz", **rec)
        manifest.append({"case": case, "fmt": fmt, "rows": rows, "cols": cols,
                         "heads": heads, "warning": bool(warning)})

    import ast
    src_path = Path(args.reference) / "sima_lmm" / "model" / "model_graph.py"
    tree = ast.parse(src_path.read_text())
    if args.only == "all":
        shapes = {"Q8_0": [(37, 64), (6, 4096)], "Q4_0": [(37, 64), (6, 4096)],
                  "Q4_K": [(37, 256), (5, 4096)], "Q5_K": [(37, 256), (5, 4096)],
                  "Q6_K": [(37, 256), (5, 4096)],
                  "Q4_1": [(37, 64), (6, 1024)], "Q5_0": [(37, 64), (6, 1024)],
                  "Q5_1": [(37, 64), (6, 1024)], "Q2_K": [(37, 256), (3, 2048)],
                  "Q3_K": [(37, 256), (3, 2048)]}
        for fmt, shp in shapes.items():
            for seed in (0, 1, 2):
                for rows, cols in shp:
                    raw = gen_tensor_bytes(fmt, rows * cols, 1000 * seed + rows)
                    run(f"{fmt}_seed{seed}_{rows}x{cols}", fmt, raw, rows, cols)
            run(f"{fmt}_single_unit", fmt, gen_tensor_bytes(fmt, FORMATS[fmt].unit_values, 77),
                1, FORMATS[fmt].unit_values)
            run(f"{fmt}_nonfinite", fmt, _nonfinite(fmt, 96 if FORMATS[fmt].unit_values == 256 else 384, 5),
                12 if FORMATS[fmt].unit_values == 256 else 48, 2048 if FORMATS[fmt].unit_values == 256 else 256)
        for fmt in ("Q4_K", "Q5_K", "Q6_K"):
            run(f"{fmt}_edges", fmt, _edge_kquant(fmt, 96, 11), 24, 1024)
        run("Q2_K_perm_q", "Q2_K", gen_tensor_bytes("Q2_K", 32 * 512, 25), 32, 512, heads=2)
        # q/k head permutation of a llama-style model: 4 heads of dim 16, and 2 kv heads
        run("Q4_K_perm_q", "Q4_K", gen_tensor_bytes("Q4_K", 64 * 512, 21), 64, 512, heads=4)
        run("Q6_K_perm_k", "Q6_K", gen_tensor_bytes("Q6_K", 32 * 512, 22), 32, 512, heads=2)
        run("Q8_0_perm_q", "Q8_0", gen_tensor_bytes("Q8_0", 64 * 128, 23), 64, 128, heads=4)
        run("F32_norm", "F32", gen_tensor_bytes("F32", 1000, 24, "norm"), 1000, 1)

        # Modalix layout: the reference's own _layout_array (model_graph.py:1271-1304), taken
        # from the source file (the module imports the absent afe SDK), applied as
        # _build_conv does (model_graph.py:1012-1042)
        fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "_layout_array")
        ns: dict = {"np": np}
        exec(compile(ast.Module(body=[fn], type_ignores=[]), str(src_path), "exec"), ns)
        layout_array = ns["_layout_array"]
        for case, (out_ch, in_ch, block) in {"layout_97x96": (97, 96, 32), "layout_64x512": (64, 512, 16)}.items():
            rng = np.random.default_rng(out_ch)
            codes = rng.integers(-128, 128, size=(out_ch, in_ch), dtype=np.int8)
            scales = rng.random((out_ch * in_ch // block, 1), dtype=np.float32)
            sc = np.transpose(np.reshape(scales, (codes.shape[0], -1)), axes=[1, 0])
            w = layout_array(layout_array(codes, "oi", "oihw"), "oihw", "hwigo")
            np.savez_compressed(out / f"{case}.npz", codes=codes, scales=scales, out_scales=sc, out_weight=w,
                                block=block, kind="layout")
            manifest.append({"case": case, "fmt": "layout", "rows": out_ch, "cols": in_ch})

    # Bundled projections: the reference's own ModelGraph._find_alternate_weight and
    # _get_array_partition (model_graph.py:1168-1248), taken from the class body the same
    # way, applied to a row-index array
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "ModelGraph")
    fns = [n for n in cls.body if isinstance(n, ast.FunctionDef)
           and n.name in ("_get_array_partition", "_find_alternate_weight")]
    pns: dict = {"np": np, "Callable": object}
    for fn_def in fns:
        fn_def.decorator_list = []   # plain functions; _find_alternate_weight names ModelGraph
    exec(compile(ast.Module(body=fns, type_ignores=[]), str(src_path), "exec"), pns)
    mgc = types.SimpleNamespace(**{f.name: pns[f.name] for f in fns})
    pns["ModelGraph"] = mgc
    part_cases = []
    for wname, q_size, kv_size, rows in [
            ("model.layers.0.self_attn.q_proj.weight", 32, 32, 9216),
            ("model.layers.0.self_attn.k_proj.weight", 32, 32, 9216),
            ("model.layers.0.self_attn.v_proj.weight", 32, 32, 9216),
            ("model.layers.3.self_attn.q_proj.weight", 24, 8, 5120),
            ("model.layers.3.self_attn.k_proj.weight", 24, 8, 5120),
            ("model.layers.3.self_attn.v_proj.weight", 24, 8, 5120),
            ("model.layers.1.mlp.gate_proj.weight", None, None, 16384),
            ("model.layers.1.mlp.up_proj.weight", None, None, 16384)]:
        fused, fn = mgc._find_alternate_weight(wname, q_size, kv_size)
        kept = fn(np.arange(rows))
        part_cases.append({"weight": wname, "q_size": q_size, "kv_size": kv_size, "rows": rows,
                           "fused": fused, "r0": int(kept[0]), "r1": int(kept[-1]) + 1})
    (out / "partition.json").write_text(json.dumps(part_cases, indent=1) + "\n")
    if args.only == "partition":
        return

    versions = {"numpy": np.__version__, "ml_dtypes": ml_dtypes.__version__,
                "gguf": getattr(gguf, "__version__", None) or _dist_version("gguf"),
                "reference": "sima-neat/llima 0.6.2", "cases": manifest}
    (out / "versions.json").write_text(json.dumps(versions, indent=1) + "\n")
    print(f"wrote {len(manifest)} cases to {out}")


def write_ggml_quant(gq, cap, out: Path, ml_dtypes, gguf):
    """Golden vectors of the reference's function-level ggml_quant API
    (``ggml_quant.py:136-886``): every unpacker, ``remove_superblocks``,
    ``convert_to_simple_block_quant`` and ``requantize_symmetric`` on seeded bytes (with
    the BASELINE distributions) and on uniform random bytes (NaN / inf / huge f16
    constants), each function's outputs stored under its own name."""
    out.mkdir(exist_ok=True)
    sym, asym = gq.QuantizationSymmetry.SYMMETRIC, gq.QuantizationSymmetry.ASYMMETRIC
    cases = []

    def u8(a):
        return a.view(np.uint8) if a.dtype in (ml_dtypes.int4, ml_dtypes.uint4) else a

    def call(rec, key, fn, *a):
        cap.messages.clear()
        with np.errstate(all="ignore"):
            res = fn(*a)
        rec[f"{key}__warning"] = "\n".join(cap.messages)
        if not isinstance(res, tuple):
            res = (res,)
        for i, r in enumerate(res):
            if r is not None:
                rec[f"{key}__{i}"] = u8(r)
                rec[f"{key}__{i}__dtype"] = str(r.dtype)
        return res

    for fmt in ("Q8_0", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"):
        f = FORMATS[fmt]
        n_units = 37 if f.unit_values == 256 else 296
        for kind in ("seed0", "seed1", "random"):
            if kind == "random":
                raw = _nonfinite(fmt, n_units, 99)
            else:
                raw = gen_tensor_bytes(fmt, n_units * f.unit_values, 500 + int(kind[-1]) * 7 + f.type_id)
            data = raw.tobytes()
            rec = {"raw": raw, "fmt": fmt}
            if fmt == "Q8_0":
                call(rec, "unpack_q8_0", gq.unpack_q8_0, data)
                call(rec, "unpack_dequantize_q8_0", gq.unpack_dequantize_q8_0, data)
                call(rec, "unpack_base_quant", gq.unpack_base_quant, data, fmt)
            elif fmt in ("Q4_0", "Q4_1"):
                s = sym if fmt == "Q4_0" else asym
                c, w = call(rec, "unpack_q4", gq.unpack_q4, data, s)
                call(rec, "unpack_dequantize_q4", gq.unpack_dequantize_q4, data, s)
                call(rec, "unpack_base_quant", gq.unpack_base_quant, data, fmt)
                if fmt == "Q4_1":
                    call(rec, "requantize_symmetric_8", gq.requantize_symmetric, c, w, 8, np.int8)
                    call(rec, "requantize_symmetric_4", gq.requantize_symmetric, c, w, 4, np.int16)
            elif fmt in ("Q5_0", "Q5_1"):
                s = sym if fmt == "Q5_0" else asym
                c, w = call(rec, "unpack_q5", gq.unpack_q5, data, s)
                call(rec, "unpack_base_quant", gq.unpack_base_quant, data, fmt)
                if fmt == "Q5_1":
                    call(rec, "requantize_symmetric_8", gq.requantize_symmetric, c, w, 8, np.int8)
                    call(rec, "requantize_symmetric_6", gq.requantize_symmetric, c, w, 6, np.int8)
            else:
                sup, blk, vals = call(rec, "unpack_k_quant", gq.unpack_k_quant, data, fmt)
                bc, q = call(rec, "remove_superblocks", gq.remove_superblocks, sup, blk, vals)
                call(rec, "remove_superblocks_f16_i16", gq.remove_superblocks, sup.astype(np.float16),
                     blk.astype(np.int16), vals)
                call(rec, "convert_to_simple_block_quant", gq.convert_to_simple_block_quant, sup, blk, vals)
                if bc.shape[1] == 2:
                    call(rec, "requantize_symmetric_5", gq.requantize_symmetric, bc.astype(np.float32), q, 5,
                         np.int32)
            np.savez_compressed(out / f"{fmt}_{kind}.npz", **rec)
            cases.append(f"{fmt}_{kind}")
    versions = {"numpy": np.__version__, "ml_dtypes": ml_dtypes.__version__,
                "gguf": getattr(gguf, "__version__", None) or _dist_version("gguf"),
                "reference": "sima-neat/llima 0.6.2", "cases": cases}
    (out / "versions.json").write_text(json.dumps(versions, indent=1) + "\n")
    print(f"wrote {len(cases)} ggml_quant cases to {out}")


def _dist_version(name: str):
    from importlib.metadata import version
    return version(name)


if __name__ == "__main__":
    main()
