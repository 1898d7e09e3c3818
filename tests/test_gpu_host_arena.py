"""Result arrays of the drop-in host calls live in the library's recycled page-locked arena.

``gguf_conversion.convert_host`` (the call ``GgufModel.load_weight`` makes through
``install()``) returns numpy arrays; from 1 MiB on they are views of page-locked buffers
from ``gq_host_alloc``, which the copy engines write directly, and a buffer goes back to the
arena when its last view is gone.  The results must not depend on where they live.
"""
import ctypes
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from llima_b200 import _native as N
from llima_b200 import gguf_conversion as G
from llima_b200.synth import gen_tensor_bytes
from oracle import ggml_oracle as O

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def _is_pinned(a: np.ndarray) -> bool:
    while a is not None and not isinstance(a, G._PinnedBlock):
        a = getattr(a, "base", None)
    return a is not None


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K", "Q8_0"])
def test_pinned_results_are_bit_exact_and_recycled(fmt):
    rows, cols = 512, 4096
    raw = gen_tensor_bytes(fmt, rows * cols, 77)
    with np.errstate(all="ignore"):
        s_ref, w_ref, _ = O.unpack_tensor(fmt, raw.tobytes(), (rows, cols), log=False)
    scales, codes, _ = G.convert_host(fmt, raw, rows, cols)
    assert _is_pinned(codes)
    assert np.array_equal(codes.view(np.uint8), w_ref.view(np.uint8))
    assert np.array_equal(scales.view(np.uint32), s_ref.view(np.uint32))
    first = codes.ctypes.data
    del scales, codes
    # the released buffer serves the next result of the same size
    scales, codes, _ = G.convert_host(fmt, raw, rows, cols)
    assert codes.ctypes.data == first
    assert np.array_equal(codes.view(np.uint8), w_ref.view(np.uint8))
    assert np.array_equal(scales.view(np.uint32), s_ref.view(np.uint32))


def test_views_keep_the_buffer():
    raw = gen_tensor_bytes("Q4_K", 256 * 4096, 5)
    _, codes, _ = G.convert_host("Q4_K", raw, 256, 4096)
    want = codes.copy()
    tail = codes[128:]
    addr = codes.ctypes.data
    del codes
    # the view still owns the buffer: a new result must not land on it
    _, other, _ = G.convert_host("Q4_K", raw, 256, 4096)
    assert other.ctypes.data != addr
    assert np.array_equal(tail, want[128:])


def test_arena_limits_and_fallback():
    lib = N.lib()
    p = ctypes.c_void_p()
    assert lib.gq_host_alloc(0, ctypes.byref(p)) == -5
    assert lib.gq_host_free(ctypes.c_void_p(12345)) == -5      # not from the arena
    assert lib.gq_host_trim() == 0
    # turned off in a fresh process: ordinary memory, same results
    code = ("import numpy as np, sys; sys.path.insert(0, %r)\n"
            "from llima_b200 import gguf_conversion as G\n"
            "from llima_b200.synth import gen_tensor_bytes\n"
            "raw = gen_tensor_bytes('Q4_K', 256 * 4096, 5)\n"
            "s, c, _ = G.convert_host('Q4_K', raw, 256, 4096)\n"
            "b = c\n"
            "while b is not None and not isinstance(b, G._PinnedBlock): b = getattr(b, 'base', None)\n"
            "assert b is None\n"
            "np.save(sys.argv[1], c)\n") % str(ROOT)
    out = Path(os.environ.get("TMPDIR", "/tmp")) / f"arena_off_{os.getpid()}.npy"
    env = dict(os.environ, LLIMA_B200_PINNED_RESULTS_MB="0")
    subprocess.run([sys.executable, "-c", code, str(out)], check=True, env=env, timeout=300)
    raw = gen_tensor_bytes("Q4_K", 256 * 4096, 5)
    _, codes, _ = G.convert_host("Q4_K", raw, 256, 4096)
    assert np.array_equal(np.load(out), codes)
    out.unlink()
