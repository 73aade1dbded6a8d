"""The allocation-free attention entry point (tcu_attend_noalloc), for callers that cannot allocate device memory
at call time - inside CUDA graph capture, under an external arena or allocator, on real-time paths. Checked
through the C ABI against the ordinary entry point (tcu_attend_device) on the same cache and queries, twice in a
row, since every call reuses the same static scratch. This file is collected last on purpose."""
import numpy as np
import pytest

from conftest import tcu
import oracle

pytestmark = pytest.mark.gpu

ATTEND = 1e-5  # attention outputs, as the other parity tests


def _case(t, kv, chunk, rows_q, seed):
    import torch
    m = t["m"]
    layers = [oracle.pack_layer(kv, m.d, t["k"][l], t["v"][l], chunk) for l in range(m.layers)]
    q = np.random.default_rng(seed).normal(0, 1, (rows_q, m.d)).astype(np.float32)
    return layers, q, torch.from_numpy(q).cuda()


def test_noalloc_attend_matches_the_allocating_entry_point(tiny):
    import torch
    t = tiny
    m = t["m"]
    gpu = tcu.Gpu(0)
    w = tcu.GpuWeights.from_bundle(gpu, t["path"])
    stream = torch.cuda.Stream()
    for call, (kv, chunk, nq) in enumerate([(1, 48, 5), (2, 37, 1), (0, 48, 32), (1, 48, 5)]):
        layers, q, qd = _case(t, kv, chunk, nq, seed=call)
        vm = tcu.VramModel.from_parts(w, [t["n"], 7, 3, chunk, kv, 1, 1], t["n"], 3, t["scales"], layers)
        for l in range(m.layers):
            want = torch.empty_like(qd)
            got = torch.full_like(qd, float("nan"))
            vm.attend_device(l, qd.data_ptr(), nq, want.data_ptr(), stream.cuda_stream)
            lay = torch.from_numpy(np.frombuffer(bytes(layers[l]), np.uint8).copy()).cuda()
            tcu.attend_noalloc(kv, m.d, m.heads, lay.data_ptr(), t["n"], chunk, qd.data_ptr(), nq, got.data_ptr(),
                               stream.cuda_stream)
            stream.synchronize()
            g, wn = got.cpu().numpy(), want.cpu().numpy()
            assert np.isfinite(g).all()
            assert np.abs(g - wn).max() < ATTEND, (call, l)
            assert np.abs(g - oracle.attend(kv, m.d, m.heads, layers[l], t["n"], chunk, q)).max() < ATTEND
        vm.free()
    w.free()
    gpu.close()


def test_noalloc_refuses_what_does_not_fit():
    import torch
    x = torch.zeros(64 * 512, device="cuda")
    with pytest.raises(tcu.TcuError) as e:
        tcu.attend_noalloc(1, 512, 4, x.data_ptr(), 100, 256, x.data_ptr(), 33, x.data_ptr())
    assert e.value.code == -1
    assert "1..32" in str(e.value)
    with pytest.raises(tcu.TcuError) as e:
        tcu.attend_noalloc(1, 512, 4, x.data_ptr(), 200000, 256, x.data_ptr(), 32, x.data_ptr())
    assert "scratch" in str(e.value)
    with pytest.raises(tcu.TcuError) as e:
        tcu.attend_noalloc(0, 512, 4, x.data_ptr(), 10 ** 6, 256, x.data_ptr(), 1, x.data_ptr())
    assert "8192" in str(e.value)
    # a misaligned pointer is refused before anything is launched (the records' scales are read as floats)
    for args in [(x.data_ptr() + 2, x.data_ptr(), x.data_ptr()), (x.data_ptr(), x.data_ptr() + 1, x.data_ptr()),
                 (x.data_ptr(), x.data_ptr(), x.data_ptr() + 6)]:
        with pytest.raises(tcu.TcuError) as e:
            tcu.attend_noalloc(1, 512, 4, args[0], 100, 256, args[1], 1, args[2])
        assert e.value.code == -1 and "aligned" in str(e.value)
