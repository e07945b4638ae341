"""The reference's own CUDA kernels against the oracle and against this library.

``oracle/_ref/libfracture_ref_kernels.so`` is built by ``make -C oracle ref``
from the reference's kernel sources (``backends/fracture-cuda/kernels/*.cu``)
with the reference's own flags (``-O3 --use_fast_math``, ``build.rs:44-56``).
Both libraries export the same C ABI (``ffi.rs:141-249``), so every case below
makes the identical ``launch_*`` call on each and compares:

* embedding, add: bit-exact, reference == oracle == this library;
* rmsnorm, rope, silu_mul: the reference's fast-math kernels are within the
  parity bar of the oracle, which pins the oracle's float statement to the
  reference implementation itself;
* TurboQuant compress: the reference kernel (tree-reduced norm, reciprocal
  multiply, fused multiply-add dot product) agrees with the exact float32
  statement on every coordinate except ones within a few 1e-7 of a decision
  boundary, where the two roundings may pick neighbouring codes; norms agree to
  within one fp16 ulp. This library reproduces the exact statement bit for bit;
* TurboQuant decompress: the reference kernel and this library decode the same
  codes to the same values within fp16 rounding.
"""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from fracture_b200 import _lib
from oracle import ops, turboquant as tq

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
REF_SO = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libfracture_ref_kernels.so"

_REF_ARGTYPES = {
    "launch_rmsnorm": [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_int, C.c_int, C.c_void_p],
    "launch_rope": [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                    C.c_void_p],
    "launch_silu_mul": [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p],
    "launch_embedding": [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p],
    "launch_add": [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p],
    "launch_turboquant_compress": [C.c_void_p] * 5 + [C.c_int] * 6 + [C.c_void_p],
    "launch_turboquant_decompress": [C.c_void_p] * 5 + [C.c_int] * 5 + [C.c_void_p],
}


@pytest.fixture(scope="module")
def libs():
    if not REF_SO.exists():
        pytest.skip("oracle/_ref not built (make -C oracle ref needs the reference sources)")
    ref = C.CDLL(str(REF_SO))
    for name, args in _REF_ARGTYPES.items():
        getattr(ref, name).argtypes = args
        getattr(ref, name).restype = C.c_int
    return {"reference": ref, "b200": _lib.load()}


def _s():
    return torch.cuda.current_stream().cuda_stream


def _h(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DEV).half()


def _np(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


def test_embedding_bit_exact_three_ways(libs):
    rng = np.random.default_rng(1)
    V, H, T = 1000, 4096, 300
    table = ops.round_to(rng.standard_normal((V, H)).astype(np.float32), "f16")
    ids = rng.integers(0, V, T).astype(np.uint32)
    ids[[5, 77]] = [V, 0xFFFFFFFF]  # out of vocabulary -> zero row
    exp = ops.embedding(table, ids)
    tt, ti = _h(table), torch.from_numpy(ids.view(np.int32)).to(DEV)
    for name, lib in libs.items():
        out = torch.full((T, H), 3.0, dtype=torch.float16, device=DEV)
        assert lib.launch_embedding(out.data_ptr(), tt.data_ptr(), ti.data_ptr(), T, H, V, _s()) == 0
        assert np.array_equal(_np(out), exp), name


def test_add_bit_exact_three_ways(libs):
    rng = np.random.default_rng(2)
    n = 3 * 4096 + 17
    a = ops.round_to(rng.standard_normal(n).astype(np.float32), "f16")
    b = ops.round_to(rng.standard_normal(n).astype(np.float32) * 3, "f16")
    exp = ops.add(a, b, "f16")
    ta, tb = _h(a), _h(b)
    for name, lib in libs.items():
        out = torch.empty(n, dtype=torch.float16, device=DEV)
        assert lib.launch_add(out.data_ptr(), ta.data_ptr(), tb.data_ptr(), n, _s()) == 0
        assert np.array_equal(_np(out), exp), name


@pytest.mark.parametrize("rows,cols", [(64, 4096), (33, 2048), (8, 256)])
def test_rmsnorm_reference_kernel_pins_oracle(libs, rows, cols):
    rng = np.random.default_rng(rows + cols)
    x = ops.round_to(rng.standard_normal((rows, cols)).astype(np.float32), "f16")
    x[:, rng.integers(0, cols, 4)] *= 20.0
    x = ops.round_to(x, "f16")
    w = ops.round_to((1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32), "f16")
    exp = ops.rmsnorm(x, w, 1e-5, "f16")
    tx, tw = _h(x), _h(w)
    got = {}
    for name, lib in libs.items():
        out = torch.empty((rows, cols), dtype=torch.float16, device=DEV)
        assert lib.launch_rmsnorm(out.data_ptr(), tx.data_ptr(), tw.data_ptr(), 1e-5, rows, cols, _s()) == 0
        got[name] = _np(out)
        ops.assert_close_fp(got[name], exp, label=f"rmsnorm {name}", dtype="f16")
    ops.assert_close_fp(got["b200"], got["reference"], label="rmsnorm b200 vs reference kernel", dtype="f16")


@pytest.mark.parametrize("T,nq,nkv,d", [(256, 32, 8, 128), (97, 4, 2, 64)])
def test_rope_reference_kernel_pins_oracle(libs, T, nq, nkv, d):
    rng = np.random.default_rng(T)
    q = ops.round_to(rng.standard_normal((T, nq, d)).astype(np.float32), "f16")
    k = ops.round_to(rng.standard_normal((T, nkv, d)).astype(np.float32), "f16")
    pos = rng.integers(0, 2048, T).astype(np.uint32)
    freqs = ops.rope_freqs(d, 10000.0)
    eq, ek = ops.rope(q, pos, freqs, "f16"), ops.rope(k, pos, freqs, "f16")
    tpos = torch.from_numpy(pos.view(np.int32)).to(DEV)
    tf = torch.from_numpy(freqs).to(DEV)
    got = {}
    for name, lib in libs.items():
        tq_, tk = _h(q), _h(k)
        assert lib.launch_rope(tq_.data_ptr(), tk.data_ptr(), tpos.data_ptr(), tf.data_ptr(), T, nq, nkv, d,
                               _s()) == 0
        got[name] = (_np(tq_), _np(tk))
        ops.assert_close_fp(got[name][0], eq, label=f"rope q {name}", dtype="f16")
        ops.assert_close_fp(got[name][1], ek, label=f"rope k {name}", dtype="f16")
    for i in range(2):
        ops.assert_close_fp(got["b200"][i], got["reference"][i], label="rope b200 vs reference kernel", dtype="f16")


def test_silu_mul_reference_kernel_pins_oracle(libs):
    rng = np.random.default_rng(9)
    n = 14336 * 8 + 5
    g = ops.round_to((rng.standard_normal(n) * 4).astype(np.float32), "f16")
    u = ops.round_to(rng.standard_normal(n).astype(np.float32), "f16")
    exp = ops.silu_mul(g, u, "f16")
    tg, tu = _h(g), _h(u)
    got = {}
    for name, lib in libs.items():
        out = torch.empty(n, dtype=torch.float16, device=DEV)
        assert lib.launch_silu_mul(out.data_ptr(), tg.data_ptr(), tu.data_ptr(), n, _s()) == 0
        got[name] = _np(out)
        ops.assert_close_fp(got[name], exp, label=f"silu_mul {name}", dtype="f16")
        assert ops.compare_tensors(got[name], exp, rtol=1e-3, atol=1e-3) == 0, name
    ops.assert_close_fp(got["b200"], got["reference"], label="silu_mul b200 vs reference kernel", dtype="f16")


def _tq_inputs(T, H, d, bits, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H, d)).astype(np.float32)
    x[rng.random(x.shape) < 0.005] *= 10.0
    x = ops.round_to(x, "f16")
    pi = tq.generate_rotation_matrix(d, 42 + bits)
    c = tq.get_codebook(d, bits).centroids.astype(np.float32)
    return x, pi, c


def _tq_compress(lib, x, pi, c, bits):
    T, H, d = x.shape
    P = tq.TurboQuantConfig.packed_dim_per_head(d, bits)
    tx, tpi, tc = _h(x), torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)
    packed = torch.zeros((T, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((T, H), dtype=torch.float16, device=DEV)
    assert lib.launch_turboquant_compress(tx.data_ptr(), tpi.data_ptr(), tc.data_ptr(), packed.data_ptr(),
                                          norms.data_ptr(), T, H, d, 1 << bits, bits, P, _s()) == 0
    torch.cuda.synchronize()
    return packed.cpu().numpy(), norms.cpu().numpy()


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("T,H,d", [(512, 8, 128), (64, 4, 64)])
def test_tq_compress_reference_kernel_pins_oracle(libs, bits, T, H, d):
    x, pi, c = _tq_inputs(T, H, d, bits, seed=T * bits + d)
    packed_exact, norms_exact, idx_exact, y_exact = tq.compress(x, pi, c, bits)
    ref_packed, ref_norms = _tq_compress(libs["reference"], x, pi, c, bits)
    ours_packed, ours_norms = _tq_compress(libs["b200"], x, pi, c, bits)

    # this library: the exact statement, bit for bit
    assert np.array_equal(ours_packed, packed_exact)
    assert np.array_equal(ours_norms.astype(np.float32), norms_exact)

    # the reference kernel: same codes except at near-ties of a decision boundary
    ref_idx = tq.unpack_indices(ref_packed.reshape(T, H, -1), bits, d)
    diff = ref_idx != idx_exact
    if diff.any():
        assert np.max(np.abs(ref_idx[diff] - idx_exact[diff])) == 1
        near = tq.boundary_distance(y_exact[diff], c)
        assert np.max(near) < 2e-6, f"reference code differs {near.max():.2e} away from a boundary"
    assert diff.mean() <= 1e-4
    # norms: the reference's tree-ordered sum and approximate sqrt move the fp16 value by at most 1 ulp
    ulp = np.abs(np.spacing(norms_exact.astype(np.float16)).astype(np.float32))
    assert np.all(np.abs(ref_norms.astype(np.float32) - norms_exact) <= ulp)
    assert np.mean(ref_norms.astype(np.float32) == norms_exact) >= 0.99


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_tq_decompress_reference_kernel_matches(libs, bits):
    T, H, d = 256, 8, 128
    x, pi, c = _tq_inputs(T, H, d, bits, seed=bits)
    packed, norms16, _, _ = tq.compress(x, pi, c, bits)
    exp = tq.decompress(packed, norms16, pi, c, bits, H, d).reshape(T, H, d)
    P = tq.TurboQuantConfig.packed_dim_per_head(d, bits)
    tp = torch.from_numpy(packed).to(DEV)
    tn = _h(norms16)
    tpi, tc = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)
    got = {}
    for name, lib in libs.items():
        out = torch.empty((T, H, d), dtype=torch.float16, device=DEV)
        assert lib.launch_turboquant_decompress(tp.data_ptr(), tn.data_ptr(), tpi.data_ptr(), tc.data_ptr(),
                                                out.data_ptr(), T, H, d, bits, P, _s()) == 0
        got[name] = _np(out)
        ops.assert_close_fp(got[name], exp, label=f"decompress {name}", dtype="f16")
    ops.assert_close_fp(got["b200"], got["reference"], label="decompress b200 vs reference kernel", dtype="f16")
