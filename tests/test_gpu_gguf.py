"""GPU: GGUF weights placed on the device by engine_gguf_load_tensor.

F32 / F16 / BF16 tensors must arrive byte for byte in row-major [N, K]; Q8_0 /
Q4_0 tensors must arrive as exactly the (payload, scales) the repack writes,
and the decode GEMV over them must match the oracle's FP64 GEMV on the file's
blocks within the derived bound.  A 32 MiB tensor crosses the 16 MiB pinned
chunks.  A type without a device layout (Q4_K) is ENGINE_ERR_UNSUPPORTED.
"""
from __future__ import annotations

import time

import numpy as np
import pytest

import oracle
from tests import bounds
from tests import gguf_writer as gw
from tests import quant_np as qn

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    rng = np.random.default_rng(2026)
    W16 = (rng.standard_normal((512, 1024)) * 0.02).astype(np.float16)
    big = (rng.standard_normal((4096, 4096)) * 0.02).astype(np.float16)   # 32 MiB
    W32 = rng.standard_normal(1024).astype(np.float32)
    bf = rng.integers(0, 2 ** 16, (64, 128), dtype=np.uint16)
    q8 = qn.quantize(qn.Q8_0, (rng.standard_normal((256, 1024)) * 0.02).astype(np.float32))
    q4 = qn.quantize(qn.Q4_0, (rng.standard_normal((300, 2048)) * 0.02).astype(np.float32))
    qk = rng.integers(0, 256, 2 * 144, dtype=np.uint8)
    tens = [("w16", gw.F16, (1024, 512), W16.tobytes()),
            ("big", gw.F16, (4096, 4096), big.tobytes()),
            ("norm", gw.F32, (1024,), W32.tobytes()),
            ("wbf", gw.BF16, (128, 64), bf.tobytes()),
            ("wq8", gw.Q8_0, (1024, 256), q8.tobytes()),
            ("wq4", gw.Q4_0, (2048, 300), q4.tobytes()),
            ("wqk", 12, (256, 2), qk.tobytes())]
    blob, _ = gw.build([("general.architecture", gw.STRING, "llama")], tens)
    path = tmp_path_factory.mktemp("gguf") / "model.gguf"
    path.write_bytes(blob)
    return path, {"w16": W16, "big": big, "norm": W32, "wbf": bf, "wq8": q8, "wq4": q4}


def test_plain_tensors_arrive_byte_for_byte(pkg, dev, model):
    path, arr = model
    with pkg.gguf.GGUFFile(path) as f:
        w16 = f.load("w16")
        assert w16.shape == (512, 1024) and w16.dtype == torch.float16
        assert np.array_equal(w16.cpu().numpy().view(np.uint16), arr["w16"].view(np.uint16))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        big = f.load("big")
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        assert np.array_equal(big.cpu().numpy().view(np.uint16), arr["big"].view(np.uint16))
        print(f"gguf load of a 32 MiB F16 tensor: {32 / 1024 / dt:.2f} GB/s (page cache warm)")
        assert np.array_equal(f.load("norm").cpu().numpy(), arr["norm"])
        wbf = f.load("wbf")
        assert wbf.dtype == torch.bfloat16
        assert np.array_equal(wbf.view(torch.int16).cpu().numpy().view(np.uint16), arr["wbf"])


@pytest.mark.parametrize("name,qt,N,K", [("wq8", qn.Q8_0, 256, 1024), ("wq4", qn.Q4_0, 300, 2048)])
def test_block_tensors_feed_the_quantised_gemv(pkg, dev, model, name, qt, N, K):
    path, arr = model
    with pkg.gguf.GGUFFile(path) as f:
        t = f.tensor(name)
        pay, sc = f.load(name)
        want_pay, want_sc = qn.split(qt, arr[name], N, K)
        assert np.array_equal(pay.cpu().numpy(), want_pay)
        assert np.array_equal(sc.cpu().numpy().view(np.uint16), want_sc.view(np.uint16))
        rng = np.random.default_rng(N)
        x = rng.standard_normal(K).astype(np.float16)
        y = pkg.ops.gemv_q(pkg.gguf.gemv_qtype(t.type), pay, sc, torch.from_numpy(x).to(dev))
        _, exact = oracle.gemv_q(qt, arr[name], x, want_f32=True)
        w = qn.dequantize(qt, arr[name], N, K).astype(np.float64)
        absdot = np.abs(w) @ np.abs(x.astype(np.float64))
        bounds.check(y.cpu().numpy().astype(np.float64), exact.astype(np.float64),
                     bounds.gemv16_bound(K, absdot, exact), f"gguf {name}")


def test_type_without_a_device_layout_is_unsupported(pkg, dev, model):
    path, _ = model
    with pkg.gguf.GGUFFile(path) as f:
        with pytest.raises(pkg.EngineError) as ei:
            f.load("wqk")
        assert ei.value.code == 3 and "GGML type 12" in str(ei.value)
