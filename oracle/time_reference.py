"""Times the reference's own CPU conversion against this repository's numpy port of it.

TEST INFRASTRUCTURE ONLY: it runs the reference (sima-neat/llima, imported from a checkout
given by --reference) and the oracle port (oracle/ggml_oracle.py) on the same seeded GGUF
bytes, in one process on one core, checks that their outputs are identical, and prints a
markdown table of GB/s of GGUF bytes per format and for the Llama-3-8B Q4_K_M format mix.
The bench's CPU baseline and reference arm time the port (the reference cannot travel to
the GPU box); this table shows what that stands for.

    python oracle/time_reference.py --reference <checkout holding sima_lmm/> [--repeats 3]
"""
from __future__ import annotations

import argparse
import platform
import sys
import time
import types
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

# (format, rows, cols): the BASELINE single-tensor shapes, and Q5_K / Q6_K at the same size
CASES = [("Q8_0", 4096, 4096), ("Q4_0", 11008, 4096), ("Q4_K", 11008, 4096), ("Q5_K", 11008, 4096),
         ("Q6_K", 11008, 4096)]


def best_of(fn, repeats: int) -> float:
    best = float("inf")
    for _ in range(repeats):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout (the directory holding sima_lmm/)")
    ap.add_argument("--repeats", type=int, default=3)
    args = ap.parse_args()
    sys.path.append(args.reference)
    sys.modules.setdefault("llama_cpp", types.SimpleNamespace(Llama=object))
    import logging
    logging.getLogger("sima_lmm.gguf.ggml_quant").setLevel(logging.ERROR)
    from gguf import GGMLQuantizationType
    from sima_lmm.gguf.gguf_conversion import unpack_gguf_tensor

    from llima_b200.synth import gen_tensor_bytes, model_specs
    from oracle import ggml_oracle as O

    rows_out = []
    rate = {}
    for fmt, rows, cols in CASES:
        raw = gen_tensor_bytes(fmt, rows * cols, 2024)
        view = types.SimpleNamespace(tensor_type=getattr(GGMLQuantizationType, fmt), data=raw, shape=[cols, rows],
                                     name=f"{fmt}_{rows}x{cols}")
        with np.errstate(all="ignore"):
            ref = unpack_gguf_tensor(view, False)
            port = O.unpack_tensor(fmt, raw, (rows, cols), log=False)[:2]
            for a, b in zip(ref, port):
                a, b = np.asarray(a), np.asarray(b)
                assert a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8)), fmt
            t_ref = best_of(lambda: unpack_gguf_tensor(view, False), args.repeats)
            t_port = best_of(lambda: O.unpack_tensor(fmt, raw, (rows, cols), log=False), args.repeats)
        rate[fmt] = (raw.size / t_ref / 1e9, raw.size / t_port / 1e9)
        rows_out.append((fmt, f"{rows}x{cols}", raw.size, t_ref, t_port))

    by_fmt: dict[str, int] = {}
    for s in model_specs("llama3-8b"):
        if s.fmt != "F32":
            by_fmt[s.fmt] = by_fmt.get(s.fmt, 0) + s.nbytes
    total = sum(by_fmt.values())
    mix_ref = total / sum(nb / (rate[f][0] * 1e9) for f, nb in by_fmt.items()) / 1e9
    mix_port = total / sum(nb / (rate[f][1] * 1e9) for f, nb in by_fmt.items()) / 1e9

    print(f"host: {platform.machine()}, numpy {np.__version__}, one process, best of {args.repeats}; "
          f"outputs of both identical bit for bit")
    print()
    print("| format | shape | GGUF MB | reference s | port s | reference GB/s | port GB/s | port / reference |")
    print("|---|---|---|---|---|---|---|---|")
    for fmt, shape, nb, tr, tp in rows_out:
        print(f"| {fmt} | {shape} | {nb / 1e6:.1f} | {tr:.3f} | {tp:.3f} | {nb / tr / 1e9:.4f} | {nb / tp / 1e9:.4f} | "
              f"{tr / tp:.2f} |")
    print(f"| Llama-3-8B Q4_K_M mix (by bytes) | | {total / 1e6:.0f} | | | {mix_ref:.4f} | {mix_port:.4f} | "
          f"{mix_port / mix_ref:.2f} |")
    return 0


if __name__ == "__main__":
    sys.exit(main())
