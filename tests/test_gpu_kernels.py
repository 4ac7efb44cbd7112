"""Kernel-level parity on the B200, through the C-ABI (libhf_cuda.so).

Config 1: the Q8_0 op sweep, W[N,K] ~ N(0, 0.02) quantized,
x[M,K] ~ N(0, 1) fp32 from seed 1, (K->N) in {2048->2048, 2048->256,
2048->16384, 16384->2048, 2048->256000} at M in {1, 8, 64}, against the
double-precision product over the dequantized weights at the reference's
dotProductTolerance(K) = 1e-5 + 2.4e-7 K (Tests/Kernels/TiledProduct.h:186-198;
LinearTests.cpp:690-715). Also the residual/gelu folds (Linear.h:205-219), the
device quantizer (byte-identical to the host), and the argmax known answers
(ArgmaxTests.cpp:107-245).
"""
import os

import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SWEEP = [(2048, 2048), (2048, 256), (2048, 16384), (16384, 2048), (2048, 256000)]


def _weights(K, N, seed=1):
    w = native.synthetic_normal(seed, 100 + N % 97, K, N * K, 0.02)
    q = native.quantize(w)
    return q, native.dequantize(q, N * K).reshape(N, K)


def _linear(x, q, K, N, M, bias=None, out=None, gelu=0, residual=0):
    lib = native.cuda()
    dq = torch.from_numpy(q).cuda()
    dx = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    dy = torch.zeros(M, N, device="cuda") if out is None else torch.from_numpy(out.copy()).cuda()
    db = None if bias is None else torch.from_numpy(bias).cuda()
    rc = lib.hf_cuda_linear_q8(dx.data_ptr(), dq.data_ptr(), None if db is None else db.data_ptr(), dy.data_ptr(),
                               K, N, M, gelu, residual, None)
    torch.cuda.synchronize()
    assert rc == 0
    return dy.cpu().numpy()


@pytest.mark.parametrize("K,N", SWEEP)
@pytest.mark.parametrize("M", [1, 8, 64])
def test_config1_op_sweep_matches_double_reference(K, N, M):
    q, deq = _weights(K, N)
    x = native.synthetic_normal(1, 200, M, M * K, 1.0).reshape(M, K)
    expected = x.astype(np.float64) @ deq.astype(np.float64).T
    got = _linear(x, q, K, N, M)
    assert ob.worst_error(got, expected) <= ob.dot_product_tolerance(K)


def _prepared(x, q, K, N, M, bias=None, out=None, gelu=False, residual=False, max_rows=64):
    """The product through a prepared weight (hf_cuda_linear_create/run)."""
    dx = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    dy = torch.zeros(M, N, device="cuda") if out is None else torch.from_numpy(out.copy()).cuda()
    db = None if bias is None else torch.from_numpy(bias).cuda()
    with native.Linear(q, K, N, max_rows) as lin:
        path = lin.path(M)
        lin.run(dx.data_ptr(), dy.data_ptr(), M, None if db is None else db.data_ptr(), gelu, residual)
        torch.cuda.synchronize()
    return dy.cpu().numpy(), path


@pytest.mark.parametrize("K,N", SWEEP)
@pytest.mark.parametrize("M", [1, 8, 64])
def test_config1_op_sweep_on_the_decoders_kernels(K, N, M):
    """The same sweep through a prepared weight, which runs the kernels the
    decoder runs: the streaming product at one row, the int8 tensor-core rows
    kernel at 8, the tcgen05 product at 64."""
    q, deq = _weights(K, N)
    x = native.synthetic_normal(1, 200, M, M * K, 1.0).reshape(M, K)
    expected = x.astype(np.float64) @ deq.astype(np.float64).T
    got, path = _prepared(x, q, K, N, M)
    assert path == {1: native.LINEAR_STREAM, 8: native.LINEAR_ROWS_MMA, 64: native.LINEAR_TENSOR_CORES}[M]
    assert ob.worst_error(got, expected) <= ob.dot_product_tolerance(K)


@pytest.mark.parametrize("M", [5, 8, 9, 16, 20, 32, 40, 64, 130])
@pytest.mark.parametrize("fold", ["bias", "gelu", "residual"])
def test_prepared_linear_folds_on_every_path(M, fold):
    K, N = 2048, 512
    q, deq = _weights(K, N, seed=6)
    x = ob.spread_values(M * K, 23 + M, 2.0).reshape(M, K)
    bias = ob.spread_values(N, 29, 1.0)
    prior = ob.spread_values(M * N, 31, 3.0).reshape(M, N)
    product = x.astype(np.float64) @ deq.astype(np.float64).T + bias
    if fold == "gelu":
        expected = np.vectorize(ob.oracle().oracle_tanh_gelu_double)(product)
        got, _ = _prepared(x, q, K, N, M, bias=bias, gelu=True, max_rows=130)
    elif fold == "residual":
        expected = product + prior
        got, _ = _prepared(x, q, K, N, M, bias=bias, out=prior, residual=True, max_rows=130)
    else:
        expected = product
        got, _ = _prepared(x, q, K, N, M, bias=bias, max_rows=130)
    assert ob.worst_error(got, expected) <= ob.dot_product_tolerance(K)


def test_prepared_linear_refusals():
    q, _ = _weights(2048, 256)
    with native.Linear(q, 2048, 256, 8) as lin:
        x = torch.zeros(9, 2048, device="cuda")
        y = torch.zeros(9, 256, device="cuda")
        with pytest.raises(native.HFError) as too_many:
            lin.run(x.data_ptr(), y.data_ptr(), 9)
        assert too_many.value.code == native.HF_E_CAPACITY
        with pytest.raises(native.HFError) as both:
            lin.run(x.data_ptr(), y.data_ptr(), 1, gelu=True, residual=True)
        assert both.value.code == native.HF_E_INVALID
    with pytest.raises(native.HFError) as shape:
        native.Linear(q[:100], 30, 10, 1)
    assert shape.value.code == native.HF_E_SHAPE


@pytest.mark.parametrize("M", [1, 3])
def test_residual_bias_and_gelu_folds(M):
    K, N = 2048, 512
    q, deq = _weights(K, N, seed=4)
    x = ob.spread_values(M * K, 17, 2.0).reshape(M, K)
    bias = ob.spread_values(N, 19, 1.0)
    prior = ob.spread_values(M * N, 23, 1.0).reshape(M, N)
    base = x.astype(np.float64) @ deq.astype(np.float64).T + bias
    got = _linear(x, q, K, N, M, bias=bias, out=prior, residual=1)
    assert ob.worst_error(got, base + prior) <= ob.dot_product_tolerance(K)
    got = _linear(x, q, K, N, M, bias=bias, gelu=1)
    expected = np.vectorize(ob.oracle().oracle_tanh_gelu_double)(base)
    assert ob.worst_error(got, expected) <= ob.dot_product_tolerance(K)


@pytest.mark.parametrize("K,N,M", [(32, 6, 2), (64, 3, 5), (2048, 384, 1), (96, 2, 4)])
def test_small_and_ragged_shapes(K, N, M):
    """LinearTests.cpp:690-715's shapes (2,32,6), (5,64,3), (1,2048,384)."""
    if (K * N) % 64:
        N += 1
    values = ob.spread_values(N * K, 31, 3.0)
    q = native.quantize(values)
    deq = native.dequantize(q, N * K).reshape(N, K)
    x = ob.spread_values(M * K, 37, 2.0).reshape(M, K)
    got = _linear(x, q, K, N, M)
    assert ob.worst_error(got, x.astype(np.float64) @ deq.astype(np.float64).T) <= ob.dot_product_tolerance(K)


def test_linear_refuses_a_shape_int8_blocks_cannot_hold():
    lib = native.cuda()
    x = torch.zeros(48, device="cuda")
    w = torch.zeros(256, dtype=torch.uint8, device="cuda")
    y = torch.zeros(4, device="cuda")
    assert lib.hf_cuda_linear_q8(x.data_ptr(), w.data_ptr(), None, y.data_ptr(), 48, 4, 1, 0, 0, None) == native.HF_E_SHAPE


def test_device_quantizer_writes_the_host_bytes():
    lib = native.cuda()
    rng = np.random.default_rng(8)
    values = (rng.standard_normal(32 * 20000) * 0.02).astype(np.float32)
    values[:32] = 0.0
    values[32:64] *= 1e-7
    values[64:96] *= 1e6
    values[96:128] = np.float32(np.inf)
    expected = native.quantize(values)
    dv = torch.from_numpy(values).cuda()
    dq = torch.zeros(expected.size, dtype=torch.uint8, device="cuda")
    half = values.size // 2
    assert lib.hf_cuda_quantize_q8(dv.data_ptr(), 0, half, values.size, dq.data_ptr(), None) == 0
    assert lib.hf_cuda_quantize_q8(dv.data_ptr() + 4 * half, half, half, values.size, dq.data_ptr(), None) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dq.cpu().numpy(), expected)


@pytest.fixture(scope="module")
def small_ctx():
    with native.Context(native.SMALL_INT8) as ctx:
        yield ctx


def test_argmax_known_answers(small_ctx):
    fixture = np.load(os.path.join(ob.GOLDEN_DIR, "reference_argmax.npz"))
    np.testing.assert_array_equal(small_ctx.argmax(fixture["hand_rows"]), fixture["hand_expected"])
    np.testing.assert_array_equal(small_ctx.argmax(fixture["spread_rows"], fixture["spread_mask"]),
                                  fixture["spread_expected"])
    vocab = ob.spread_values(256000, 256000, 4.0)
    vocab[137425] = 900.0
    vocab[318] = 800.0
    mask = np.zeros(256000, dtype=np.float32)
    assert small_ctx.argmax(vocab)[0] == 137425
    mask[137425] = 1.0
    assert small_ctx.argmax(vocab, mask)[0] == 318
    last = ob.spread_values(256000, 4242, 4.0)
    last[-1] = 900.0
    assert small_ctx.argmax(last)[0] == 255999
    survivor = np.full(37, 1.0, dtype=np.float32)
    survivor[11] = 0.0
    row = (1000.0 - np.arange(37)).astype(np.float32)
    row[11] = -1000.0
    assert small_ctx.argmax(row, survivor)[0] == 11
    assert small_ctx.argmax(row, np.ones(37, dtype=np.float32))[0] == 0


def test_argmax_ties_take_the_lowest_index(small_ctx):
    rng = np.random.default_rng(12)
    rows = rng.integers(-3, 3, (16, 5000)).astype(np.float32)
    expected = [ob.argmax(r) for r in rows]
    np.testing.assert_array_equal(small_ctx.argmax(rows), expected)
