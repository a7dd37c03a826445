"""Engine semantics on the B200 that newch callers rely on: the error model, host-visible data
(mirrors), memory release during backward and at step end, checkpoints, optimizer state access,
gradient checks, the C-side modules, and integer-exact int8 layers."""

from __future__ import annotations

import ctypes
import os
import tempfile

import numpy as np
import pytest

from nchelp import Eng, capi, rel_err, seeded
import ncoracle as O

pytestmark = pytest.mark.gpu
ALL = capi.ALL_AXES


def test_backend_and_device():
    with Eng() as e:
        assert e.L.nc_kernel_backend(e.ctx) == b"b200"
        assert e.L.nc_ext_device_count() >= 1
        assert b"B200" in e.L.nc_ext_device_name(e.ctx) or e.L.nc_ext_device_name(e.ctx)


def test_shape_error_is_sticky_and_null_propagates():
    with Eng() as e:
        a, b = e.t(np.zeros((2, 3), np.float32)), e.t(np.zeros((4, 5), np.float32))
        assert not e.L.nc_add(a, b)
        assert e.L.nc_status_code(e.ctx) == 1 and b"broadcast" in e.L.nc_error(e.ctx)
        assert not e.L.nc_relu(None)
        assert not e.L.nc_relu(a)  # sticky: ops refuse while an error is pending
        e.L.nc_clear_error(e.ctx)
        assert e.L.nc_relu(a)


def test_dtype_error_then_retry_like_newch_promotion():
    with Eng() as e:
        i = e.t(np.arange(4, dtype=np.int32))
        assert not e.L.nc_scale(i, 2.0) and e.L.nc_status_code(e.ctx) == 2
        e.L.nc_clear_error(e.ctx)
        f = e.check(e.L.nc_to_dtype(i, capi.F32))
        assert np.array_equal(e.np(e.check(e.L.nc_scale(f, 2.0))), np.arange(4) * 2.0)


def test_label_out_of_range_is_an_argument_error():
    with Eng() as e:
        x = e.param(seeded(1, (3, 4)))
        assert not e.L.nc_cross_entropy(x, e.t(np.array([0, 4, 1], np.int32)))
        assert e.L.nc_status_code(e.ctx) == 4


def test_device_side_label_check_reports_at_sync():
    """Labels computed on the device (no host copy) are checked by the kernel: the error surfaces at
    the next synchronization instead of faulting."""
    with Eng() as e:
        x = e.param(seeded(2, (3, 4)))
        lab_f = e.t(np.array([0.0, 9.0, 1.0], np.float32))
        lab = e.check(e.L.nc_to_dtype(e.check(e.L.nc_scale(lab_f, 1.0)), capi.I32))  # device-made labels
        loss = e.L.nc_cross_entropy(x, lab)
        assert loss  # enqueued
        v = e.L.nc_item(loss)
        assert e.L.nc_status_code(e.ctx) == 4, (v, e.err())


def test_data_f32_mirror_round_trip():
    with Eng() as e:
        x = e.param(np.arange(6, dtype=np.float32))
        p = e.L.nc_data_f32(x)
        arr = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)), shape=(6,))
        assert np.array_equal(arr, np.arange(6))
        arr[2] = 100.0  # host write through the pointer reaches the device before the next op
        y = e.np(e.check(e.L.nc_scale(x, 1.0)))
        assert y[2] == 100.0


def test_item_get_copy():
    with Eng() as e:
        x = e.t(np.arange(12, dtype=np.float32).reshape(3, 4))
        t = e.check(e.L.nc_transpose(x, 0, 1))
        n, idx = capi.shape_arg((3, 1))
        assert e.L.nc_get(t, idx) == 7.0
        assert e.L.nc_item(e.check(e.L.nc_sum(x, ALL, 0))) == 66.0
        assert np.array_equal(e.np(t), np.arange(12, dtype=np.float32).reshape(3, 4).T)


def test_backward_releases_memory_and_step_end_resets():
    with Eng() as e:
        w = e.param(seeded(3, (256, 256)))
        x = e.t(seeded(4, (512, 256)))
        h = x
        for _ in range(6):
            h = e.check(e.L.nc_relu(e.check(e.L.nc_linear_fn(h, w, None))))
        loss = e.check(e.L.nc_mean(h, ALL, 0))
        before = e.L.nc_get_mem_stats(e.ctx).arena_bytes_in_use
        assert e.L.nc_backward_ex(loss, 1, None, 0) == 0
        after = e.L.nc_get_mem_stats(e.ctx).arena_bytes_in_use
        assert after < before
        assert e.grad(w) is not None
        e.step_end()
        assert e.L.nc_get_mem_stats(e.ctx).arena_bytes_in_use == 0


def test_second_backward_through_released_graph_fails():
    with Eng() as e:
        w = e.param(seeded(5, (4, 4)))
        y = e.check(e.L.nc_sum(e.check(e.L.nc_tanh(e.check(e.L.nc_linear_fn(e.t(seeded(6, (3, 4))), w, None)))),
                               ALL, 0))
        assert e.L.nc_backward_ex(y, 1, None, 0) == 0
        assert e.L.nc_backward_ex(y, 1, None, 0) == 5


def test_retain_graph_accumulates():
    with Eng() as e:
        w = e.param(seeded(7, (4,)))
        y = e.check(e.L.nc_sum(e.check(e.L.nc_mul(w, w)), ALL, 0))
        assert e.L.nc_backward_ex(y, 2, None, 0) == 0
        assert e.L.nc_backward_ex(y, 2, None, 0) == 0
        assert np.allclose(e.grad(w), 4 * e.np(w), rtol=1e-6)


def test_save_load_round_trip():
    with Eng() as e:
        a = e.param(seeded(8, (3, 5)))
        b = e.t(np.arange(7, dtype=np.int32), persistent=True)
        path = os.path.join(tempfile.mkdtemp(), "t.ncw")
        names = (ctypes.c_char_p * 2)(b"a", b"b")
        ts = capi.ptr_array([a, b])
        assert e.L.nc_save(e.ctx, path.encode(), 2, names, ts) == 0
        a2 = e.param(np.zeros((3, 5), np.float32))
        b2 = e.t(np.zeros(7, np.int32), persistent=True)
        assert e.L.nc_load(e.ctx, path.encode(), 2, names, capi.ptr_array([a2, b2])) == 0
        assert np.array_equal(e.np(a2), e.np(a)) and np.array_equal(e.np(b2), np.arange(7))
        raw = open(path, "rb").read()
        assert raw[:4] == b"NCW1"


def _ncw1_items():
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    from make_ncw1 import OUT, ncw1_tensors

    return OUT, ncw1_tensors()


def test_ncw1_written_by_the_reference_loads():
    """tests/golden/ref_state.ncw was written by the reference engine's nc_save (make_ncw1.py)."""
    path, items = _ncw1_items()
    with Eng() as e:
        ts = [e.t(np.zeros_like(a), persistent=True) for _, a in items]
        names = (ctypes.c_char_p * len(items))(*[n.encode() for n, _ in items])
        assert e.L.nc_load(e.ctx, str(path).encode(), len(items), names, capi.ptr_array(ts)) == 0, e.err()
        for (n, a), t in zip(items, ts):
            assert np.array_equal(e.np(t), a), n


def test_ncw1_written_here_matches_the_reference_bytes():
    path, items = _ncw1_items()
    with Eng() as e:
        ts = [e.t(a, persistent=True) for _, a in items]
        names = (ctypes.c_char_p * len(items))(*[n.encode() for n, _ in items])
        out = os.path.join(tempfile.mkdtemp(), "b200.ncw")
        assert e.L.nc_save(e.ctx, out.encode(), len(items), names, capi.ptr_array(ts)) == 0, e.err()
    assert open(out, "rb").read() == path.read_bytes()


def _resume_model(e, W1, B1, W2):
    ps = [e.param(W1), e.param(B1), e.param(W2)]
    opt = e.check(e.L.nc_adamw(e.ctx, capi.ptr_array(ps), 3, capi.OptimOpts(1e-2, 0.0, 0.01, 0.9, 0.999, 1e-8)))
    return ps, opt


def _resume_step(e, ps, opt, X, Y):
    e.L.nc_optim_clear_grad(opt)
    h = e.check(e.L.nc_relu(e.check(e.L.nc_linear_fn(e.t(X), ps[0], ps[1]))))
    loss = e.check(e.L.nc_cross_entropy(e.check(e.L.nc_linear_fn(h, ps[2], None)), e.t(Y)))
    assert e.L.nc_backward(loss) == 0, e.err()
    e.L.nc_optim_step(opt)
    e.step_end()


def test_bit_exact_resume_from_checkpoint():
    """Train 3 steps, checkpoint the parameters (NCW1) and the optimizer state (state pointers and
    step count, as newch's Optimizer.state_dict does), then 3 more steps; a fresh context restored
    from the checkpoint takes the same 3 steps to bit-identical parameters (newch
    tests/test_checkpoint.py:57-73)."""
    rng = np.random.default_rng(5)
    W1, B1, W2 = (rng.standard_normal(s).astype(np.float32) * 0.3 for s in ((16, 12), (16,), (5, 16)))
    batches = [(rng.standard_normal((32, 12)).astype(np.float32), rng.integers(0, 5, 32).astype(np.int32))
               for _ in range(6)]
    path = os.path.join(tempfile.mkdtemp(), "ckpt.ncw")
    names = (ctypes.c_char_p * 3)(b"w1", b"b1", b"w2")
    with Eng() as e:
        ps, opt = _resume_model(e, W1, B1, W2)
        for X, Y in batches[:3]:
            _resume_step(e, ps, opt, X, Y)
        assert e.L.nc_save(e.ctx, path.encode(), 3, names, capi.ptr_array(ps)) == 0
        state = [[np.frombuffer(ctypes.string_at(e.L.nc_optim_state(opt, i, s), 4 * W.size), np.float32).copy()
                  for s in (0, 1)] for i, W in enumerate((W1, B1, W2))]
        step = e.L.nc_optim_get_step(opt)
        for X, Y in batches[3:]:
            _resume_step(e, ps, opt, X, Y)
        straight = [e.np(p) for p in ps]
        e.L.nc_optim_free(opt)
    with Eng() as e:
        ps, opt = _resume_model(e, np.zeros_like(W1), np.zeros_like(B1), np.zeros_like(W2))
        assert e.L.nc_load(e.ctx, path.encode(), 3, names, capi.ptr_array(ps)) == 0, e.err()
        for i, st in enumerate(state):
            for s, arr in enumerate(st):
                ctypes.memmove(e.L.nc_optim_state(opt, i, s), arr.ctypes.data, arr.nbytes)
        e.L.nc_optim_set_step(opt, step)
        for X, Y in batches[3:]:
            _resume_step(e, ps, opt, X, Y)
        resumed = [e.np(p) for p in ps]
        e.L.nc_optim_free(opt)
    for a, b in zip(straight, resumed):
        assert np.array_equal(a, b)


def test_optimizer_state_pointer_round_trip():
    """newch/optim.py reads the state with ctypes.string_at and writes it with memmove."""
    with Eng() as e:
        w = e.param(seeded(9, (10,)))
        opt = e.check(e.L.nc_adam(e.ctx, capi.ptr_array([w]), 1, capi.OptimOpts(0.1, 0, 0, 0, 0, 0)))
        e.L.nc_optim_clear_grad(opt)
        assert e.L.nc_backward(e.check(e.L.nc_sum(e.check(e.L.nc_mul(w, w)), ALL, 0))) == 0
        e.L.nc_optim_step(opt)
        m = e.L.nc_optim_state(opt, 0, 0)
        mv = np.frombuffer(ctypes.string_at(m, 40), np.float32).copy()
        g = 2 * seeded(9, (10,))
        assert rel_err(mv, 0.1 * g) < 1e-6
        ctypes.memmove(m, np.zeros(10, np.float32).ctypes.data, 40)  # load_state_dict writes it
        v = e.L.nc_optim_state(opt, 0, 1)
        ctypes.memmove(v, np.ones(10, np.float32).ctypes.data, 40)
        w_before = e.np(w)
        e.step_end()
        e.L.nc_optim_clear_grad(opt)
        assert e.L.nc_backward(e.check(e.L.nc_sum(e.check(e.L.nc_scale(w, 0.0)), ALL, 0))) == 0
        e.L.nc_optim_step(opt)  # zero grad, m = 0, v = 1: w moves by lr * 0 = 0 (m uploaded)
        assert np.allclose(e.np(w), w_before)
        e.L.nc_optim_free(opt)


def test_gradient_accumulation_gate():
    with Eng() as e:
        w = e.param(np.ones(3, np.float32))
        opt = e.check(e.L.nc_sgd(e.ctx, capi.ptr_array([w]), 1, capi.OptimOpts(0.5, 0, 0, 0, 0, 0)))
        e.L.nc_optim_set_accumulation(opt, 2)
        for k in range(2):
            e.L.nc_optim_zero_grad(opt)
            assert e.L.nc_backward(e.check(e.L.nc_sum(w, ALL, 0))) == 0
            e.L.nc_optim_step(opt)
            e.step_end()
            if k == 0:
                assert np.array_equal(e.np(w), np.ones(3))
        assert np.allclose(e.np(w), 0.5)  # averaged grad 1, lr 0.5
        assert e.L.nc_optim_get_step(opt) == 1


def test_clip_grad_norm():
    with Eng() as e:
        w = e.param(np.array([3.0, 4.0], np.float32))
        assert e.L.nc_backward(e.check(e.L.nc_sum(e.check(e.L.nc_mul(w, e.t(np.array([3.0, 4.0], np.float32)))),
                                                  ALL, 0))) == 0
        norm = e.L.nc_clip_grad_norm(capi.ptr_array([w]), 1, 1.0)
        assert norm == pytest.approx(5.0)
        assert np.allclose(e.grad(w), [0.6, 0.8], rtol=1e-5)


def test_gradcheck_conv_and_bn():
    with Eng() as e:
        fn_t = capi.SCALAR_FN

        @fn_t
        def f(ctx, inputs, user):
            y = e.L.nc_conv2d(inputs[0], inputs[1], None, 1, 1, 1, 1)
            return e.L.nc_sum(e.L.nc_tanh(y), ALL, 0)

        ins = capi.ptr_array([e.param(seeded(10, (1, 2, 4, 4), 0.5)), e.param(seeded(11, (2, 2, 3, 3), 0.5))])
        err = e.L.nc_gradcheck(e.ctx, f, ins, 2, None, 1e-2)
        assert err < 2e-2, err


def test_c_modules():
    with Eng(seed=5) as e:
        mods = capi.ptr_array([e.L.nc_linear(e.ctx, 4, 8, 1), e.L.nc_act(e.ctx, 0), e.L.nc_linear(e.ctx, 8, 2, 1)])
        seq = e.check(e.L.nc_sequential(e.ctx, 3, mods))
        assert e.L.nc_module_name(seq) == b"Sequential"
        out = (ctypes.c_void_p * 8)()
        assert e.L.nc_parameters(seq, out, 8) == 4
        y = e.check(e.L.nc_forward(seq, e.t(seeded(12, (5, 4)))))
        assert e.shape(y) == (5, 2)


def test_int8_layer_bit_exact_against_reference():
    """linear_int8 on identical inputs: quantization, int32 accumulators and the rescale all exact."""
    w, x, b = seeded(20, (96, 257), 0.2), seeded(21, (33, 257)), seeded(22, (96,))
    outs = []
    for which in ("b200", "ref"):
        with Eng(which) as e:
            sp = capi.ptr_array([None])
            q = e.check(e.L.nc_quantize_rows(e.t(w), sp))
            y = e.check(e.L.nc_linear_int8(e.t(x), q, sp[0], e.t(b)))
            outs.append((e.np(q), e.np(sp[0]), e.np(y)))
    for a, r in zip(*outs):
        assert np.array_equal(a, r)
    yo, acc, _, _ = O.linear_int8(x, outs[1][0], outs[1][1], b)
    assert np.array_equal(outs[0][2], yo)


@pytest.mark.parametrize("path", ["tc", "dp4a"])
@pytest.mark.parametrize("M,N,K", [(512, 1024, 1024), (300, 200, 1040), (129, 130, 256), (64, 64, 64), (40, 700, 96)])
def test_int8_gemm_paths_bit_exact(path, M, N, K, monkeypatch):
    """The int8 GEMM on tcgen05 (kind::i8, exact int32 accumulation; K in 128-byte steps with the TMA's
    zero fill past K) and on dp4a: quantization, outputs and the rescale equal the reference's bit for
    bit. Shapes: cfg5-like, ragged M / N / K tails, one partial K step."""
    monkeypatch.setenv("NC_QGEMM", path)
    w, x, b = seeded(30, (N, K), 0.2), seeded(31, (M, K)), seeded(32, (N,))
    outs = []
    for which in ("b200", "ref"):
        with Eng(which) as e:
            sp = capi.ptr_array([None])
            q = e.check(e.L.nc_quantize_rows(e.t(w), sp))
            y = e.check(e.L.nc_linear_int8(e.t(x), q, sp[0], e.t(b)))
            outs.append((e.np(q), e.np(sp[0]), e.np(y)))
    for a, r in zip(*outs):
        assert np.array_equal(a, r)
    yo, _, _, _ = O.linear_int8(x, outs[1][0], outs[1][1], b)
    assert np.array_equal(outs[0][2], yo)


@pytest.mark.parametrize("jump", ["poly", "matrix"])
@pytest.mark.parametrize("n", [1, 31, 16384, 16385, 100000, 1 << 20, (1 << 21) + 77, 3 << 20])
def test_dropout_masks_match_reference_stream(n, jump, monkeypatch):
    """Device jump-ahead reproduces the reference stream for any length, and the host stream
    continues where the kernel stopped. Both jump kernels: by run polynomials (the default) and by
    jump matrices (NC_DROPOUT_JUMP=matrix; the path for tensors beyond the polynomial table)."""
    monkeypatch.setenv("NC_DROPOUT_JUMP", jump)
    res = []
    for which in ("b200", "ref"):
        with Eng(which, seed=99) as e:
            x = e.t(np.ones(n, np.float32))
            y1 = e.np(e.check(e.L.nc_dropout(x, 0.3)))
            y2 = e.np(e.check(e.L.nc_dropout(x, 0.7)))
            n1, shp = capi.shape_arg((5,))
            u = e.np(e.check(e.L.nc_rand_uniform(e.ctx, 0.0, 1.0, n1, shp)))
            res.append((y1, y2, u))
    for a, b in zip(*res):
        assert np.array_equal(a, b)


def test_empty_and_scalar_tensors():
    with Eng() as e:
        z = e.t(np.zeros((0, 5), np.float32))
        assert e.shape(e.check(e.L.nc_relu(z))) == (0, 5)
        s = e.check(e.L.nc_sum(z, ALL, 0))
        assert e.L.nc_item(s) == 0.0
        m = e.check(e.L.nc_mean(z, ALL, 0))
        assert np.isnan(e.L.nc_item(m))
        sc = e.check(e.L.nc_scalar(e.ctx, 2.5))
        assert e.L.nc_item(sc) == 2.5


def test_persistent_and_release():
    with Eng() as e:
        before = e.L.nc_get_mem_stats(e.ctx).persistent_bytes
        p = e.param(np.ones((1000,), np.float32))
        assert e.L.nc_is_persistent(p)
        assert e.L.nc_get_mem_stats(e.ctx).persistent_bytes >= before + 4000
        e.L.nc_release(p)
        assert e.L.nc_get_mem_stats(e.ctx).persistent_bytes == before
