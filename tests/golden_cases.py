"""Loader for the golden vectors written by tests/golden/make_golden.py."""
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def case_names(prefix: str = "") -> list[str]:
    """Golden cases of the GGUF conversion (the layout cases are listed by layout_cases)."""
    return sorted(p.stem for p in GOLDEN.glob(f"{prefix}*.npz") if not p.stem.startswith("layout_"))


def layout_cases() -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob("layout_*.npz"))


def load_case(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as z:
        rec = {k: z[k] for k in z.files}
    for k in ("rows", "cols", "perm_heads"):
        if k in rec:
            rec[k] = int(rec[k])
    rec["fmt"] = str(rec["fmt"])
    rec["warning"] = str(rec["warning"])
    rec["codes_dtype"] = str(rec["codes_dtype"])
    return rec


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit equality, with every NaN equal to every other NaN (payloads are not compared)."""
    a = np.asarray(a)
    b = np.asarray(b)
    if a.shape != b.shape:
        return False
    if a.dtype.kind == "f":
        a32 = a.astype(np.float32)
        b32 = b.astype(np.float32)
        nan = np.isnan(a32) & np.isnan(b32)
        return bool(np.all(nan | (a32.view(np.uint32) == b32.view(np.uint32))))
    return bool(np.array_equal(a.view(np.uint8), b.view(np.uint8)))
