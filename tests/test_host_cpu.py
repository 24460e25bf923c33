"""Host-side logic of the seam, without a GPU: value types, output validation, the loader
contract the reference probes (runtime/native.py), and the camera partition."""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from shipinfer_b200 import NormalizeParams, check_device_output
from shipinfer_b200.errors import ConfigurationError, ValidationError

needs_no_gpu = pytest.mark.skipif(torch.cuda.is_available(), reason="checks the GPU-less behaviour")


def test_normalize_params_mirror_the_reference():
    p = NormalizeParams()
    assert p.mean == (0.0, 0.0, 0.0) and p.std == (255.0, 255.0, 255.0) and p.swap_rb is True
    with pytest.raises(ValueError, match="non-zero"):
        NormalizeParams(std=(1.0, 0.0, 1.0))


def test_output_validation_messages():
    with pytest.raises(ValidationError, match="needs a CUDA tensor"):
        check_device_output(torch.empty(1, 3, 8, 8), device_index=0, rows=1, caller="letterbox_to_device")

    class Fake:  # a CUDA-looking tensor on another device
        is_cuda = True
        device = torch.device("cpu")

    fake = Fake()
    fake.device = type("D", (), {"index": 1})()
    with pytest.raises(ValidationError, match="cross-device"):
        check_device_output(fake, device_index=0, rows=1, caller="x")


@needs_no_gpu
def test_native_ops_refuse_a_host_without_b200():
    from shipinfer_b200 import NativeImageOps

    with pytest.raises(ConfigurationError, match="no usable GPU kernels"):
        NativeImageOps(device_index=0)


def test_shipvision_surface_as_the_reference_loader_reads_it():
    """runtime/native.py:47-150: import by name, `cuda_available` probe, `__version__` and
    `platform` attributes (platform is a string, not a call), `device_count()`."""
    from shipinfer_b200 import shipvision_C

    shipvision_C.install()
    try:
        module = importlib.import_module("shipvision._C")
        assert module is shipvision_C
        probe = getattr(module, "cuda_available", None)
        assert callable(probe) and isinstance(probe(), bool)
        assert isinstance(module.__version__, str) and module.__version__
        assert isinstance(module.platform, str) and not callable(module.platform)
        assert isinstance(module.device_count(), int)
        assert hasattr(module, "ImageOps")
    finally:
        import sys

        sys.modules.pop("shipvision._C", None)
        sys.modules.pop("shipvision", None)


def test_camera_partition_rules():
    from shipinfer_b200.shard import plan_cameras, shard_of

    load = {"a": 30.0, "b": 30.0, "c": 5.0, "d": 5.0, "e": 5.0}
    plan = plan_cameras(load, [0, 1])
    assert sorted(sum(plan, ())) == sorted(load) and plan == [("a", "c", "e"), ("b", "d")]
    assert shard_of(load, [0, 1], 1) == ("b", "d")
    with pytest.raises(ConfigurationError):
        plan_cameras(load, [])
    with pytest.raises(ConfigurationError):
        plan_cameras({"a": 1.0}, [0, 1])


def test_oracle_handles_empty_and_degenerate_inputs():
    from oracle import oracle

    assert oracle.nms(np.zeros((0, 4), np.float32), np.zeros(0, np.float32), 0.5, 0.0, 10).size == 0
    keep, counts = oracle.nms_batched(np.zeros((2, 0, 4), np.float32), np.zeros((2, 0), np.float32), None,
                                      0.5, 0.0, 5, class_aware=False)
    assert (keep == -1).all() and counts.tolist() == [0, 0]
    crops = oracle.crop([np.full((4, 4, 3), 9, np.uint8)], np.array([[1, 1, 1, 3]], np.float32), (2, 2),
                        None, (1.0, 2.0, 3.0), (2.0, 2.0, 2.0), True)
    assert np.array_equal(crops[0, :, 0, 0], np.array([-0.5, -1.0, -1.5], np.float32))
