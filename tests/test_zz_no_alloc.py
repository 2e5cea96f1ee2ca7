"""The allocation-free decode attention entry point (needs a B200).

hyc_attention_decode_noalloc serves callers that cannot allocate device
memory where they call it — a host whose own arena or caching allocator holds
all free device memory, or a serving loop that must not let cudaMalloc /
cudaFree synchronise the device.  It keeps its split-KV scratch in a fixed
file-scope device array instead.  This test calls it through the C ABI on
device buffers the test owns, twice in a row (the second call reuses the
scratch the first one left behind), and checks each result against the
allocating entry point (hyc_attention_test) on the same inputs, with the
tolerance the attention parity tests use.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# the scratch holds kv_heads * ceil(ctx / 128) * group * (hdim + 2) floats
SCRATCH_FLOATS, SPLIT = 131072, 128


def _rope(lib, hd, ctx):
    cos = np.zeros(ctx * (hd // 2), dtype=np.float32)
    sin = np.zeros_like(cos)
    assert lib.hyc_rope_tables(10000.0, 1000.0, hd, hd, ctx, cos.ctypes.data, sin.ctypes.data) == 0
    return cos, sin


def _bf16(x):
    return (np.asarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _geometry(hd, group):
    """The fewest KV heads (a power of two, at least 2) whose largest context
    the fixed scratch accepts is at most 64 splits, and that context."""
    kvh = 2
    while SCRATCH_FLOATS // (kvh * group * (hd + 2)) > 64:
        kvh *= 2
    return kvh, SCRATCH_FLOATS // (kvh * group * (hd + 2)) * SPLIT


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("group", [1, 2, 4, 8])
def test_noalloc_attention_matches_allocating_entry_point(hd, group):
    """Every (hdim, group) the entry point dispatches, at a position inside
    the first 128 keys (one split: the output is written without the
    scratch), mid-context, and at the last position of the largest context
    the scratch limit allows; each as two calls in a row (pos, pos + 1) so
    the second call starts from the scratch contents the first one left."""
    import torch

    from hymt2_b200.device import Backend

    kvh, ctx = _geometry(hd, group)
    heads = kvh * group
    be = Backend(0)
    lib = be.lib
    try:
        rng = np.random.default_rng(2024 + hd + group)
        qd, kvd = heads * hd, kvh * hd
        cos, sin = _rope(lib, hd, ctx)
        qn = (1.0 + 0.2 * rng.standard_normal(hd)).astype(np.float32)
        kn = (1.0 + 0.2 * rng.standard_normal(hd)).astype(np.float32)
        kc = _bf16(rng.standard_normal((ctx, kvd)))
        vc = _bf16(rng.standard_normal((ctx, kvd)))

        dev = torch.device("cuda", 0)
        d_kc = torch.from_numpy(kc.view(np.int16).copy()).to(dev)
        d_vc = torch.from_numpy(vc.view(np.int16).copy()).to(dev)
        d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
        d_qn, d_kn = torch.from_numpy(qn).to(dev), torch.from_numpy(kn).to(dev)
        d_ao = torch.zeros(qd, dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev)
        err = ctypes.create_string_buffer(256)

        for pos in (37, 38, 300, 301, ctx - 2, ctx - 1):
            qkv = (rng.standard_normal((1, qd + 2 * kvd)) * 2.0).astype(np.float32)
            # allocating entry point on host copies of the same cache state
            kc_ref, vc_ref = d_kc.cpu().numpy().view(np.uint16).copy(), d_vc.cpu().numpy().view(np.uint16).copy()
            want = be.attention_test(heads, kvh, hd, ctx, qkv, pos, kc_ref, vc_ref, qn, kn, cos, sin)
            d_qkv = torch.from_numpy(qkv.reshape(-1).copy()).to(dev)
            d_pos = torch.tensor([pos], dtype=torch.int32, device=dev)
            rc = lib.hyc_attention_decode_noalloc(
                ctypes.c_void_p(stream.cuda_stream), heads, kvh, hd, ctx, d_pos.data_ptr(), 1e-5, d_qkv.data_ptr(),
                d_kc.data_ptr(), d_vc.data_ptr(), d_qn.data_ptr(), d_kn.data_ptr(), d_cos.data_ptr(),
                d_sin.data_ptr(), d_ao.data_ptr(), err, 256)
            assert rc == 0, err.value.decode()
            torch.cuda.synchronize(dev)
            got = d_ao.cpu().numpy()[None]
            rel = np.abs(got - want).max() / max(np.abs(want).max(), 1e-6)
            assert rel < 1e-4, (hd, group, pos, rel)
            kc_got, vc_got = d_kc.cpu().numpy().view(np.uint16), d_vc.cpu().numpy().view(np.uint16)
            assert np.array_equal(vc_got[pos], vc_ref[pos]) and np.array_equal(kc_got[pos], kc_ref[pos])

        # one split more than the fixed scratch holds is refused with a clear error
        big = (SCRATCH_FLOATS // (kvh * group * (hd + 2)) + 1) * SPLIT
        rc = lib.hyc_attention_decode_noalloc(
            ctypes.c_void_p(stream.cuda_stream), heads, kvh, hd, big, d_pos.data_ptr(), 1e-5, d_qkv.data_ptr(),
            d_kc.data_ptr(), d_vc.data_ptr(), d_qn.data_ptr(), d_kn.data_ptr(), d_cos.data_ptr(), d_sin.data_ptr(),
            d_ao.data_ptr(), err, 256)
        assert rc == -2 and b"scratch limit" in err.value
    finally:
        be.close()
