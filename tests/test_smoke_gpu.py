"""smoke_fill and build_info on the GPU (the reference's tests/test_smoke_kernel.py,
tests/test_build_info.py and the device half of tests/test_cuda_extension.py)."""
import math
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DTYPES = [torch.float64, torch.float32, torch.float16, torch.bfloat16]


@pytest.fixture(scope="module")
def ext():
    from decode_llm_kernel_b200 import cuda
    cuda.require()
    return cuda


@pytest.mark.parametrize("dtype", DTYPES)
def test_fills_every_element(ext, dtype):
    x = torch.zeros(1024, dtype=dtype, device="cuda")
    ext.smoke_fill(x, 3.5)
    torch.cuda.synchronize()
    assert torch.equal(x, torch.full_like(x, 3.5))


@pytest.mark.parametrize("value", [0.0, 1.0, -2.25, 3.5, 256.0])
def test_writes_the_requested_value(ext, value):
    x = torch.ones(97, dtype=torch.float32, device="cuda")
    ext.smoke_fill(x, value)
    torch.cuda.synchronize()
    assert torch.equal(x, torch.full_like(x, value))


def test_double_tensor_keeps_double_precision(ext):
    x = torch.zeros(64, dtype=torch.float64, device="cuda")
    ext.smoke_fill(x, math.pi)
    torch.cuda.synchronize()
    assert torch.equal(x, torch.full_like(x, math.pi))


@pytest.mark.parametrize("shape", [(1,), (7,), (255,), (256,), (257,), (4, 8, 16), (1, 1, 1)])
def test_shapes_that_do_not_divide_the_block_size(ext, shape):
    x = torch.zeros(shape, dtype=torch.float32, device="cuda")
    ext.smoke_fill(x, 1.0)
    torch.cuda.synchronize()
    assert int((x != 1.0).sum()) == 0


def test_grid_stride_loop_covers_more_than_one_pass(ext):
    x = torch.zeros(20_000_000, dtype=torch.bfloat16, device="cuda")
    ext.smoke_fill(x, 2.0)
    torch.cuda.synchronize()
    assert int((x != 2.0).sum()) == 0


def test_empty_and_return_value(ext):
    x = torch.empty(0, dtype=torch.float32, device="cuda")
    assert ext.smoke_fill(x, 1.0) is None
    backing = torch.zeros(1024, dtype=torch.float32, device="cuda")
    ext.smoke_fill(backing[:100], 9.0)
    torch.cuda.synchronize()
    assert int(backing[100:].abs().sum()) == 0 and bool((backing[:100] == 9.0).all())


def test_rejections(ext):
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ext.smoke_fill(torch.zeros(4), 1.0)
    with pytest.raises(RuntimeError, match="contiguous"):
        ext.smoke_fill(torch.zeros(8, 8, device="cuda")[:, ::2], 1.0)
    with pytest.raises(RuntimeError, match="not implemented"):
        ext.smoke_fill(torch.zeros(4, dtype=torch.int32, device="cuda"), 1.0)


def test_non_default_stream_and_graph_capture(ext):
    x = torch.zeros(4096, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ext.smoke_fill(x, 4.0)
    torch.cuda.synchronize()
    assert int((x != 4.0).sum()) == 0
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ext.smoke_fill(x, 7.0)
    x.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(x, torch.full_like(x, 7.0))


def test_build_info(ext):
    info = ext.build_info()
    for key in ("gencode_arch", "cuda_version_compiled", "cuda_version_runtime",
                "cuda_version_driver", "nvcc_version", "fast_math"):
        assert key in info
    major, minor = torch.cuda.get_device_capability(0)
    assert int(info["gencode_arch"]) == major * 100 + minor * 10
    assert info["fast_math"] == "0"
    assert info["cuda_version_compiled"] == ".".join(info["nvcc_version"].split(".")[:2])
    assert info["cuda_version_runtime"] == torch.version.cuda


def test_loads_without_the_caller_importing_torch_first():
    probe = subprocess.run(
        [sys.executable, "-c",
         "from decode_llm_kernel_b200 import cuda; print(cuda.is_available())"],
        cwd=ROOT, capture_output=True, text=True)
    assert probe.stdout.strip() == "True", probe.stdout + probe.stderr


def test_launch_floor_probe_runs(ext):
    ext.require().launch_empty(4, False)
    ext.require().launch_empty(4, True)
    torch.cuda.synchronize()
