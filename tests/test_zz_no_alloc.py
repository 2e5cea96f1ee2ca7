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

HEADS, KVH, HD, CTX = 16, 4, 128, 1024


def _rope(lib):
    cos = np.zeros(CTX * (HD // 2), dtype=np.float32)
    sin = np.zeros_like(cos)
    assert lib.hyc_rope_tables(10000.0, 1000.0, HD, HD, CTX, cos.ctypes.data, sin.ctypes.data) == 0
    return cos, sin


def _bf16(x):
    return (np.asarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_noalloc_attention_matches_allocating_entry_point():
    import torch

    from hymt2_b200.device import Backend

    be = Backend(0)
    lib = be.lib
    try:
        rng = np.random.default_rng(2024)
        qd, kvd = HEADS * HD, KVH * HD
        cos, sin = _rope(lib)
        qn = (1.0 + 0.2 * rng.standard_normal(HD)).astype(np.float32)
        kn = (1.0 + 0.2 * rng.standard_normal(HD)).astype(np.float32)
        kc = np.zeros((CTX, kvd), dtype=np.uint16)
        vc = np.zeros((CTX, kvd), dtype=np.uint16)
        kc[:300] = _bf16(rng.standard_normal((300, kvd)))
        vc[:300] = _bf16(rng.standard_normal((300, kvd)))

        dev = torch.device("cuda", 0)
        d_kc = torch.from_numpy(kc.view(np.int16).copy()).to(dev)
        d_vc = torch.from_numpy(vc.view(np.int16).copy()).to(dev)
        d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
        d_qn, d_kn = torch.from_numpy(qn).to(dev), torch.from_numpy(kn).to(dev)
        d_ao = torch.zeros(qd, dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev)
        err = ctypes.create_string_buffer(256)

        for pos in (300, 301):          # two calls in a row; 3 splits each (scratch in use)
            qkv = (rng.standard_normal((1, qd + 2 * kvd)) * 2.0).astype(np.float32)
            # allocating entry point on host copies of the same cache state
            kc_ref, vc_ref = d_kc.cpu().numpy().view(np.uint16).copy(), d_vc.cpu().numpy().view(np.uint16).copy()
            want = be.attention_test(HEADS, KVH, HD, CTX, qkv, pos, kc_ref, vc_ref, qn, kn, cos, sin)
            d_qkv = torch.from_numpy(qkv.reshape(-1).copy()).to(dev)
            d_pos = torch.tensor([pos], dtype=torch.int32, device=dev)
            rc = lib.hyc_attention_decode_noalloc(
                ctypes.c_void_p(stream.cuda_stream), HEADS, KVH, HD, CTX, d_pos.data_ptr(), 1e-5, d_qkv.data_ptr(),
                d_kc.data_ptr(), d_vc.data_ptr(), d_qn.data_ptr(), d_kn.data_ptr(), d_cos.data_ptr(),
                d_sin.data_ptr(), d_ao.data_ptr(), err, 256)
            assert rc == 0, err.value.decode()
            torch.cuda.synchronize(dev)
            got = d_ao.cpu().numpy()[None]
            rel = np.abs(got - want).max() / max(np.abs(want).max(), 1e-6)
            assert rel < 1e-4, (pos, rel)
            kc_got, vc_got = d_kc.cpu().numpy().view(np.uint16), d_vc.cpu().numpy().view(np.uint16)
            assert np.array_equal(vc_got[pos], vc_ref[pos]) and np.array_equal(kc_got[pos], kc_ref[pos])

        # a shape beyond the fixed scratch is refused with a clear error
        rc = lib.hyc_attention_decode_noalloc(
            ctypes.c_void_p(stream.cuda_stream), 64, 64, 128, 65536, d_pos.data_ptr(), 1e-5, d_qkv.data_ptr(),
            d_kc.data_ptr(), d_vc.data_ptr(), d_qn.data_ptr(), d_kn.data_ptr(), d_cos.data_ptr(), d_sin.data_ptr(),
            d_ao.data_ptr(), err, 256)
        assert rc == -2 and b"scratch limit" in err.value
    finally:
        be.close()
