"""The VM's MATVEC and FFN opcodes on the GPU against the reference's
arithmetic restated in numpy over the oracle's exact decoders: M = 1 in the
matvec orientation (W[i + j*K]), M > 1 and FFN in the row-major [K, N]
reading of the dequantised W, the bias rules of exec_ffn."""
import numpy as np
import pytest

from oracle import oracle as O
from m3_avm_b200 import synth

pytestmark = pytest.mark.gpu


def dense(raw, dtype, n):
    if dtype == 0:
        return np.frombuffer(np.ascontiguousarray(raw).tobytes(), np.float32)[:n].astype(np.float64)
    if dtype == 1:
        return np.frombuffer(np.ascontiguousarray(raw).tobytes(), np.float16)[:n].astype(np.float64)
    return O.dequantize(raw, dtype, n).astype(np.float64)


def weights(dtype, K, N, seed):
    if dtype in (0, 1):
        a = (synth.activations(K * N, seed) * np.float32(0.1)).astype(np.float32 if dtype == 0 else np.float16)
        return a.view(np.uint8).reshape(-1)
    return synth.weights(dtype, K, N, seed)


@pytest.fixture(scope="module")
def T():
    import torch

    from m3_avm_b200 import _lib

    _lib.load()
    return lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("dtype", [12, 14, 8, 2, 0, 1])
@pytest.mark.parametrize("M", [1, 3, 17])
def test_matvec_opcode(T, dtype, M):
    import torch

    from m3_avm_b200 import vm_ops

    K, N = 512, 768
    raw = weights(dtype, K, N, 10 + dtype)
    W = dense(raw, dtype, K * N)
    X = synth.activations(K, 11, batch=M)
    y = vm_ops.exec_matvec(T(X if M > 1 else X[0]), T(raw), dtype, K, N)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    if M == 1:
        Wm = W.reshape(N, K)  # matvec orientation: W[i + j*K]
        want = (Wm @ X[0].astype(np.float64))[None, :]
        scale = np.abs(Wm) @ np.abs(X[0].astype(np.float64))
    else:
        Wm = W.reshape(K, N)  # row-major reading of exec_matvec's ndarray path
        want = X.astype(np.float64) @ Wm
        scale = np.abs(X.astype(np.float64)) @ np.abs(Wm)
    assert np.all(np.abs(got - want) <= 1e-5 * scale + 1e-6), np.max(np.abs(got - want) / (scale + 1e-30))


@pytest.mark.parametrize("bias", ["none", "broadcast", "per_row", "wrong_length"])
def test_ffn_opcode(T, bias):
    import torch

    from m3_avm_b200 import vm_ops

    M, D, H, Do = 5, 256, 512, 256
    w1 = synth.weights(12, D, H, 21)
    w2 = synth.weights(14, H, Do, 22)
    W1 = dense(w1, 12, D * H).reshape(D, H)
    W2 = dense(w2, 14, H * Do).reshape(H, Do)
    X = synth.activations(D, 23, batch=M) * np.float32(0.05)
    b1 = b2 = None
    B1 = np.zeros((M, H))
    B2 = np.zeros((M, Do))
    if bias == "broadcast":
        b1, b2 = synth.activations(H, 24), synth.activations(Do, 25)
        B1, B2 = np.broadcast_to(b1, (M, H)), np.broadcast_to(b2, (M, Do))
    elif bias == "per_row":
        b1, b2 = synth.activations(H, 24, batch=M), synth.activations(Do, 25, batch=M)
        B1, B2 = b1, b2
    elif bias == "wrong_length":
        b1, b2 = synth.activations(H + 1, 24), synth.activations(3, 25)
    hidden = X.astype(np.float64) @ W1 + B1
    with np.errstate(over="ignore"):
        gated = hidden / (1.0 + np.exp(-hidden))
    want = gated @ W2 + B2
    y = vm_ops.exec_ffn(T(X), T(w1), 12, H, T(w2), 14, Do, b1=T(b1) if b1 is not None else None,
                        b2=T(b2) if b2 is not None else None)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    scale = np.abs(gated) @ np.abs(W2) + (np.abs(X.astype(np.float64)) @ np.abs(W1)) @ np.abs(W2) * 1e-2
    assert np.all(np.abs(got - want) <= 1e-4 * scale + 1e-5), np.max(np.abs(got - want) / (scale + 1e-30))


def test_opcode_rules(T):
    from m3_avm_b200 import _lib, vm_ops

    with pytest.raises(_lib.M3GError):  # x cols != W rows
        vm_ops.exec_matvec(T(np.zeros((2, 256), np.float32)), T(synth.weights(12, 512, 256, 1)), 12, 512, 256)
    with pytest.raises(_lib.M3GError):  # W shorter than K*N
        vm_ops.exec_matvec(T(np.zeros((2, 512), np.float32)), T(synth.weights(12, 256, 256, 1)), 12, 512, 256)
