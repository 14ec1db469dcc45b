"""torch.ops.batch_topk_b200.{topk, topk_segmented}: the custom-operator registration over the
C ABI.  The fake (shape-only) kernels are checked on the CPU; the GPU tests compare the
operator with the oracle (bit-exact), with torch.topk (values), and under torch.compile."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import batch_topk_b200.torch_api  # noqa: F401  (registers the operators)
from batch_topk_b200 import workloads as wl
from util import assert_exact


def test_fake_kernels_give_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty((7, 1000), dtype=torch.float16, device="cuda")
        v, i = torch.ops.batch_topk_b200.topk(x, 13)
        assert v.shape == (7, 13) and v.dtype == torch.float16
        assert i.shape == (7, 13) and i.dtype == torch.int32
        off = torch.empty((9,), dtype=torch.int32, device="cuda")
        x1 = torch.empty((5000,), dtype=torch.float16, device="cuda")
        v, i = torch.ops.batch_topk_b200.topk_segmented(x1, off, 4)
        assert v.shape == (8, 4) and i.shape == (8, 4)


def test_fake_kernel_rejects_wrong_dtype():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode(), pytest.raises(ValueError):
        torch.ops.batch_topk_b200.topk(torch.empty((2, 10), dtype=torch.float64, device="cuda"), 3)


def test_fake_kernels_keep_bfloat16():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty((3, 500), dtype=torch.bfloat16, device="cuda")
        v, i = torch.ops.batch_topk_b200.topk(x, 7)
        assert v.shape == (3, 7) and v.dtype == torch.bfloat16 and i.dtype == torch.int32
        off = torch.empty((4,), dtype=torch.int32, device="cuda")
        v, i = torch.ops.batch_topk_b200.topk_segmented(torch.empty((900,), dtype=torch.bfloat16,
                                                                    device="cuda"), off, 5)
        assert v.shape == (3, 5) and v.dtype == torch.bfloat16


def test_fake_kernels_keep_float32():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty((3, 500), dtype=torch.float32, device="cuda")
        v, i = torch.ops.batch_topk_b200.topk(x, 7)
        assert v.shape == (3, 7) and v.dtype == torch.float32 and i.dtype == torch.int32


def test_eager_calls_reject_host_tensors_and_other_dtypes():
    from batch_topk_b200 import torch_api

    with pytest.raises(ValueError):
        torch_api.topk(torch.zeros((2, 10), dtype=torch.float16), 3)       # host memory
    with pytest.raises(ValueError):
        torch_api.topk(torch.zeros((2, 10), dtype=torch.float64), 3)       # no float64 path
    with pytest.raises(ValueError):
        torch_api.topk_segmented(torch.zeros((10,), dtype=torch.bfloat16),
                                 torch.zeros((3,), dtype=torch.int32), 2)


@pytest.mark.gpu
def test_operator_matches_oracle_and_torch_topk(orc):
    x = wl.gen_c2(rows=slice(0, 16))
    xt = torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16)
    v, i = torch.ops.batch_topk_b200.topk(xt, 50)
    exp_v, exp_i = orc.topk(x, 50)
    assert_exact(v.cpu().view(torch.int16).numpy().view(np.uint16), i.cpu().numpy(), exp_v, exp_i,
                 "op vs oracle")
    tv, _ = torch.topk(xt, 50, dim=1)  # values agree; torch's order among ties is unspecified
    assert torch.equal(v, tv)
    assert torch.equal(torch.gather(xt, 1, i.long()), v)


@pytest.mark.gpu
def test_operator_under_torch_compile(orc):
    x = wl.gen_c1()
    xt = torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16)

    def f(t):
        v, i = torch.ops.batch_topk_b200.topk(t * 2, 50)
        return v.float().sum(dim=1), i

    g = torch.compile(f, fullgraph=True)
    s_ref, i_ref = f(xt)
    s_cmp, i_cmp = g(xt)
    assert torch.equal(i_ref, i_cmp) and torch.equal(s_ref, s_cmp)


@pytest.mark.gpu
def test_segmented_operator(orc):
    rng = np.random.default_rng(3)
    lens = np.array([0, 5, 100, 20000, 7, 70000])
    off = np.zeros(lens.size + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    vals = rng.standard_normal(int(off[-1])).astype(np.float16).view(np.uint16)
    xt = torch.from_numpy(vals.view(np.int16)).cuda().view(torch.float16)
    ot = torch.from_numpy(off.astype(np.int32)).cuda()
    v, i = torch.ops.batch_topk_b200.topk_segmented(xt, ot, 50)
    exp_v, exp_i = orc.topk_csr(vals, off, 50)
    assert_exact(v.cpu().view(torch.int16).numpy().view(np.uint16), i.cpu().numpy(), exp_v, exp_i,
                 "segmented op vs oracle")


@pytest.mark.gpu
def test_two_explicit_streams_get_separate_workspaces(orc):
    """Calls on two explicit streams under one current stream each use the default workspace
    of their own launch stream, so overlapping calls do not race on a shared buffer."""
    import torch

    from batch_topk_b200.torch_api import topk

    dev = torch.device("cuda:0")
    rng = np.random.default_rng(31)
    a = rng.standard_normal((256, 151936)).astype(np.float16)
    b = rng.standard_normal((256, 151936)).astype(np.float16)
    xa = torch.from_numpy(a).to(dev)
    xb = torch.from_numpy(b).to(dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s1.wait_stream(torch.cuda.current_stream(dev))
    s2.wait_stream(torch.cuda.current_stream(dev))
    outs = []
    for _ in range(3):
        outs.append(topk(xa, 50, stream=s1) + (a,))
        outs.append(topk(xb, 50, stream=s2) + (b,))
    torch.cuda.synchronize(dev)
    for v, i, src in outs:
        exp_v, exp_i = orc.topk(src.view(np.uint16), 50)
        assert np.array_equal(i.cpu().numpy(), exp_i)
        assert np.array_equal(v.cpu().numpy().view(np.uint16), exp_v)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_input_on_another_device_than_the_current_one(orc):
    """x on cuda:1 while cuda:0 is current: the call runs on x's device."""
    from batch_topk_b200.torch_api import topk

    rng = np.random.default_rng(32)
    a = rng.standard_normal((64, 40000)).astype(np.float16)
    with torch.cuda.device(0):
        x = torch.from_numpy(a).to("cuda:1")
        v, i = topk(x, 50)
        assert v.device == x.device and i.device == x.device
        torch.cuda.synchronize(1)
    exp_v, exp_i = orc.topk(a.view(np.uint16), 50)
    assert np.array_equal(i.cpu().numpy(), exp_i)
    assert np.array_equal(v.cpu().numpy().view(np.uint16), exp_v)
