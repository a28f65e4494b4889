"""Generate the golden vectors that pin the CPU oracle to the reference.

Run where the reference source tree (bnb_jax 0.2.0) is available, giving its
root directory (the one that holds ``src/bnb_jax``)::

    python tests/golden/make_golden.py <reference-root>

The reference (bnb_jax 0.2.0) is pure Python over JAX, cutejax and the CUTLASS
DSL, none of which can run here. Its host-side functions, however, are plain
Python/numpy once those imports are stubbed:

* ``kernels/quantize.py:53-88``  ``create_dynamic_map``      (numpy, exact)
* ``kernels/quantize.py:46-50``  ``_NF4_THRESHOLDS``         (constants)
* ``kernels/quantize.py:91-95``  ``_quantize_nf4``           (code selection)
* ``kernels/quantize.py:102-125`` ``_quantize_8bit``         (code selection)
* ``kernels/dequantize.py:27-32`` ``NF4_TABLE``               (constants)
* ``kernels/dequantize.py:87-90`` ``_log2_blocksize``         (validation)
* ``kernels/gemv.py:42``, ``:207-215`` ``GEMV_MAX_M``, ``_rows_per_warp``

The stubs give the DSL scalar types numpy float32 / Python int semantics, so
``_quantize_nf4`` and ``_quantize_8bit`` execute the reference's own
comparison code on float32 values. Their outputs on a large set of scaled
values (every threshold and midpoint, +-k ulp, random values, specials) are
stored in ``reference_golden.npz`` and checked against the oracle by
``tests/test_oracle_golden.py``. The GPU box never runs this script.
"""
from __future__ import annotations

import importlib
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _install_stubs() -> None:
    """Replace jax / cutejax / cutlass with the minimum the reference's
    module bodies touch at import time, and scalar semantics for the two
    code-selection functions."""
    jnp = types.ModuleType("jax.numpy")
    jnp.float16 = np.float16
    jnp.float32 = np.float32
    jnp.bfloat16 = "bfloat16"
    jnp.uint8 = np.uint8
    jnp.dtype = lambda d: d if isinstance(d, str) else np.dtype(d)
    jnp.array = lambda data, dtype=None: np.array(data, dtype=dtype)
    jnp.asarray = lambda data, dtype=None: np.asarray(data, dtype=dtype)
    jnp.zeros = lambda shape, dtype=None: np.zeros(shape, dtype=dtype)

    jax = types.ModuleType("jax")
    jax.numpy = jnp
    jax.Array = object

    class _CustomVJP:
        def __init__(self, f):
            self.f = f

        def defvjp(self, fwd, bwd):
            self.fwd, self.bwd = fwd, bwd

        def __call__(self, *a, **k):
            return self.f(*a, **k)

    jax.custom_vjp = _CustomVJP
    tree_util = types.ModuleType("jax.tree_util")
    tree_util.register_dataclass = lambda cls: cls
    jax.tree_util = tree_util
    jax.tree = types.SimpleNamespace(leaves=lambda t: [], map=None)
    jax.ShapeDtypeStruct = lambda *a, **k: None

    cutejax = types.ModuleType("cutejax")
    cutejax.call = None
    cutejax.ArraySpec = lambda **k: None

    cutlass = types.ModuleType("cutlass")
    cutlass.Int32 = lambda v: int(v)
    cutlass.Float32 = lambda v: np.float32(v)
    cutlass.select_ = lambda c, a, b: a if c else b
    cutlass.Constexpr = type("Constexpr", (), {"__class_getitem__": classmethod(lambda c, i: c)})
    cute = types.ModuleType("cutlass.cute")
    cute.kernel = lambda f: f
    cute.jit = lambda f: f
    cute.Tensor = object
    arch = types.ModuleType("cutlass.cute.arch")
    arch.inline_ptx = None
    cute.arch = arch
    cutlass.cute = cute

    sys.modules.update({
        "jax": jax, "jax.numpy": jnp, "jax.tree_util": tree_util,
        "cutejax": cutejax, "cutlass": cutlass, "cutlass.cute": cute,
        "cutlass.cute.arch": arch,
    })


def _load_reference(root: Path):
    if not (root / "src" / "bnb_jax" / "kernels" / "quantize.py").is_file():
        raise SystemExit(f"{root} is not the reference's root (no src/bnb_jax/kernels/quantize.py)")
    _install_stubs()
    sys.path.insert(0, str(root / "src"))
    q = importlib.import_module("bnb_jax.kernels.quantize")
    d = importlib.import_module("bnb_jax.kernels.dequantize")
    g = importlib.import_module("bnb_jax.kernels.gemv")
    return q, d, g


def _ulp_neighbours(vals: np.ndarray, k: int) -> np.ndarray:
    out = [vals]
    up = vals.copy()
    dn = vals.copy()
    for _ in range(k):
        up = np.nextafter(up, np.float32(np.inf))
        dn = np.nextafter(dn, np.float32(-np.inf))
        out += [up, dn]
    return np.concatenate(out).astype(np.float32)


def main(argv: list[str]) -> None:
    if len(argv) != 1:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference-root>")
    q, d, g = _load_reference(Path(argv[0]))
    rng = np.random.default_rng(20261201)

    thresholds = np.array(q._NF4_THRESHOLDS, np.float32)
    table = np.asarray(d.NF4_TABLE, np.float32)
    dmap = np.asarray(q.create_dynamic_map(), np.float32)
    dmap_unsigned = np.asarray(q.create_dynamic_map(signed=False), np.float32)
    dmap_4bit = np.asarray(q.create_dynamic_map(max_exponent_bits=3, total_bits=4), np.float32)

    # scaled values (x * r) the NF4 code selection sees
    specials = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan,
                         1.0000001, -1.0000001, 1e-30, -1e-30], np.float32)
    nf4_in = np.concatenate([
        _ulp_neighbours(thresholds, 3),
        _ulp_neighbours(table, 2),
        specials,
        rng.uniform(-1.0, 1.0, 20000).astype(np.float32),
        (rng.standard_normal(5000) * 0.3).astype(np.float32),
    ])
    nf4_out = np.array([q._quantize_nf4(np.float32(v)) for v in nf4_in], np.uint8)

    # 8-bit code selection against the dynamic map and a user codebook
    mids = ((dmap[1:] + dmap[:-1]) * np.float32(0.5)).astype(np.float32)
    q8_in = np.concatenate([
        _ulp_neighbours(dmap, 2),
        _ulp_neighbours(mids, 2),
        specials,
        rng.uniform(-1.0, 1.0, 20000).astype(np.float32),
        (rng.standard_normal(5000) * 0.05).astype(np.float32),
        np.sign(rng.standard_normal(4000)).astype(np.float32)
        * np.power(np.float32(10.0), rng.uniform(-8, 0, 4000)).astype(np.float32),
    ])
    q8_out = np.array([q._quantize_8bit(dmap, np.float32(v)) for v in q8_in], np.uint8)

    user_code = np.sort(rng.uniform(-1.0, 1.0, 256).astype(np.float32))
    user_code[0], user_code[-1] = -1.0, 1.0
    umids = ((user_code[1:] + user_code[:-1]) * np.float32(0.5)).astype(np.float32)
    q8u_in = np.concatenate([_ulp_neighbours(umids, 2), _ulp_neighbours(user_code, 1),
                             specials, rng.uniform(-1.05, 1.05, 10000).astype(np.float32)])
    q8u_out = np.array([q._quantize_8bit(user_code, np.float32(v)) for v in q8u_in], np.uint8)

    log2_ok = {bs: d._log2_blocksize(bs) for bs in (8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096)}
    log2_bad = []
    for bs in (0, 4, 7, 48, 100, 3000):
        try:
            d._log2_blocksize(bs)
        except ValueError:
            log2_bad.append(bs)

    np.savez_compressed(
        HERE / "reference_golden.npz",
        nf4_thresholds=thresholds,
        nf4_table=table,
        dynamic_map=dmap,
        dynamic_map_unsigned=dmap_unsigned,
        dynamic_map_4bit=dmap_4bit,
        nf4_code_in=nf4_in, nf4_code_out=nf4_out,
        q8_code_in=q8_in, q8_code_out=q8_out,
        q8_user_code=user_code, q8_user_in=q8u_in, q8_user_out=q8u_out,
        log2_blocksizes=np.array(sorted(log2_ok)), log2_values=np.array([log2_ok[b] for b in sorted(log2_ok)]),
        log2_rejected=np.array(log2_bad),
        gemv_max_m=np.array(g.GEMV_MAX_M),
        rows_per_warp=np.array([g._rows_per_warp(m) for m in range(1, 21)]),
    )
    print(f"wrote {HERE / 'reference_golden.npz'}: {len(nf4_in)} nf4 cases, "
          f"{len(q8_in)} + {len(q8u_in)} 8-bit cases")


if __name__ == "__main__":
    main(sys.argv[1:])
