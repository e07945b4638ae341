"""fb_launch_tq_compress_paged_noalloc against fb_launch_tq_compress_paged, through the C ABI.

The no-allocation entry point runs the same launch sequence as the paged entry
point (whose exact-settle queue lives in each CTA's shared memory), with a
per-call vector limit, so its pool bytes and norms must equal the paged entry
point's bit for bit. Two calls in a row with different inputs check that no
state carries over between calls. The file sorts last so that it also runs
after every other GPU test in one process.
"""

import numpy as np
import pytest
import torch

from fracture_b200 import _lib
from fracture_b200 import kernels as K
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MAX_VECTORS = 1 << 19
TDT = {"f16": torch.float16, "bf16": torch.bfloat16}
FBT = {"f16": _lib.FB_FP16, "bf16": _lib.FB_BF16}


def _inputs(T, H, d, dt, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H, d)).astype(np.float32)
    x[rng.random(x.shape) < 0.005] *= 10.0
    return torch.from_numpy(ops.round_to(x, dt)).to(DEV).to(TDT[dt])


def _paged(T, start_pos, seed):
    """Shuffled block table covering positions [0, start_pos + T) of a pool with spare blocks."""
    nblk = (start_pos + T + 15) // 16
    pool_blocks = nblk + 5
    rng = np.random.default_rng(seed)
    table = rng.permutation(pool_blocks)[:nblk].astype(np.int32)
    return torch.from_numpy(table).to(DEV), pool_blocks * 16


def _outputs(rows, H, d, bits):
    packed = torch.full((rows, H * (d * bits // 8)), 0xA5, dtype=torch.uint8, device=DEV)
    norms = torch.full((rows, H), 7.0, dtype=torch.float16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    return packed, norms, err


def _call(fn_name, x, dt, pi, c, bits, table, start_pos, rows, out=None):
    T, H, d = x.shape
    packed, norms, err = out if out is not None else _outputs(rows, H, d, bits)
    rc = getattr(_lib.load(), fn_name)(
        x.data_ptr(), FBT[dt], pi.data_ptr(), c.data_ptr(), bits, T, H, d,
        table.data_ptr() if table is not None else None, start_pos, rows, packed.data_ptr(), norms.data_ptr(),
        err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, (fn_name, rc, _lib.load().fb_last_error())
    return packed, norms, err


def _tables(d, bits, seed):
    c, _ = K.tq_codebook(d, bits)
    pi = K.tq_rotation_matrix(d, seed)
    return torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("bits", [2, 3, 4])
def test_noalloc_matches_allocating_entry_two_calls(dt, bits):
    H, d = 8, 128
    pi, c = _tables(d, bits, 42 + bits)
    for call, (T, start_pos) in enumerate([(4099, 37), (2048, 0)]):
        x = _inputs(T, H, d, dt, seed=1000 * bits + call)
        table, rows = _paged(T, start_pos, seed=call)
        ref = _call("fb_launch_tq_compress_paged", x, dt, pi, c, bits, table, start_pos, rows)
        got = _call("fb_launch_tq_compress_paged_noalloc", x, dt, pi, c, bits, table, start_pos, rows)
        torch.cuda.synchronize()
        assert torch.equal(got[0], ref[0]), f"packed differs on call {call}"
        assert torch.equal(got[1].view(torch.int16), ref[1].view(torch.int16)), f"norms differ on call {call}"
        assert int(got[2].item()) == int(ref[2].item()) == 0


def test_noalloc_max_size_and_no_device_allocation():
    """A call at the limit matches the paged entry point; calls after the first leave free device memory unchanged."""
    H, d, bits, dt = 8, 128, 4, "f16"
    T = MAX_VECTORS // H
    pi, c = _tables(d, bits, 7)
    x = _inputs(T, H, d, dt, seed=3)
    outs = [_outputs(T, H, d, bits) for _ in range(2)]
    _call("fb_launch_tq_compress_paged_noalloc", x, dt, pi, c, bits, None, 0, T, out=outs[1])  # loads the module
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for o in outs:
        o[0].fill_(0xA5)
        _call("fb_launch_tq_compress_paged_noalloc", x, dt, pi, c, bits, None, 0, T, out=o)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] >= free0 - (2 << 20)
    ref = _call("fb_launch_tq_compress_paged", x, dt, pi, c, bits, None, 0, T)
    torch.cuda.synchronize()
    for got in outs:
        assert torch.equal(got[0], ref[0])
        assert torch.equal(got[1].view(torch.int16), ref[1].view(torch.int16))


def test_noalloc_rejects_oversize_before_launch():
    lib = _lib.load()
    H, d, bits = 8, 128, 4
    T = MAX_VECTORS // H + 1
    # no buffer is touched: the size check comes before any pointer is used
    dummy = torch.zeros(16, dtype=torch.uint8, device=DEV)
    p = dummy.data_ptr()
    rc = lib.fb_launch_tq_compress_paged_noalloc(p, _lib.FB_FP16, p, p, bits, T, H, d, None, 0, T, p, p, None,
                                                 torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    msg = lib.fb_last_error().decode()
    assert "per-call limit" in msg and str(MAX_VECTORS) in msg
    torch.cuda.synchronize()


def test_noalloc_exact_path_shapes_match():
    """head_dim other than 128 and 8-bit codes take the CUDA-core path."""
    for (T, H, d, bits) in [(33, 8, 64, 4), (40, 4, 128, 8)]:
        pi, c = _tables(d, bits, 11)
        x = _inputs(T, H, d, "f16", seed=T)
        ref = _call("fb_launch_tq_compress_paged", x, "f16", pi, c, bits, None, 0, T)
        got = _call("fb_launch_tq_compress_paged_noalloc", x, "f16", pi, c, bits, None, 0, T)
        torch.cuda.synchronize()
        assert torch.equal(got[0], ref[0]) and torch.equal(got[1].view(torch.int16), ref[1].view(torch.int16))

