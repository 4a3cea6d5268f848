"""Device-side failure reporting: bounded waits that give up, and V values a bf16 cache cannot hold.

No test here faults or hangs the GPU.  A wait is made to run out on an
mbarrier that nothing arrives on, with a short poll limit; the kernel returns
and the host reads the flag through nmg_device_status.
"""
import ctypes

import pytest
import torch

from hero_b200 import _lib, nm

pytestmark = pytest.mark.gpu


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


@pytest.mark.parametrize("target", [0, 1])
def test_a_wait_that_runs_out_is_reported_once(dev, target):
    nm.device_status(0)  # start clean
    _lib.call("nmg_selftest_wait_timeout", 0, target, _stream(dev))
    with pytest.raises(_lib.DeviceTimeout):
        nm.device_status(0)
    nm.device_status(0)  # reported and cleared: the next call is clean
    # the context is still usable afterwards
    assert torch.ones(4, device=dev).sum().item() == 4


def test_status_is_clean_without_failures(dev):
    cache = nm.FullAttentionCache(2, 128, capacity=64, dtype="bf16")
    x = torch.randn(64, 256, device=dev).bfloat16()
    cache.append(0, x, x)
    nm.attend(cache, torch.randn(1, 4 * 128, device=dev).bfloat16(), 63, 0.1)
    nm.device_status(0)


@pytest.mark.parametrize("src", [torch.float32, torch.bfloat16])
def test_bf16_cache_reports_v_beyond_fp16(dev, src):
    # A bf16 cache keeps V as fp16 (largest finite 65504): a value that rounds
    # to bf16 magnitude 65536 or more cannot be held and is reported; values
    # just inside the range, and K of any size, are fine.
    nm.device_status(0)
    cache = nm.FullAttentionCache(1, 64, capacity=8, dtype="bf16")
    k = torch.full((2, 64), 1e6, device=dev).to(src)
    v = torch.full((2, 64), 65280.0, device=dev).to(src)  # the largest bf16 below 65504
    cache.append(0, k, v)
    nm.device_status(0)
    assert float(cache.value(1, 0)[0]) == 65280.0
    v_big = torch.zeros(1, 64, device=dev).to(src)
    v_big[0, 17] = -70000.0
    cache.append(2, k[:1], v_big)
    with pytest.raises(_lib.ValueOverflow):
        nm.device_status(0)
    assert float(cache.value(2, 0)[17]) == float("-inf")
    nm.device_status(0)


def test_bf16_prologue_reports_v_beyond_fp16(dev):
    # The attention prologue writes V straight into the cache with the same rule.
    nm.device_status(0)
    hq, hkv, dh, T = 2, 1, 64, 4
    cache = nm.FullAttentionCache(hkv, dh, capacity=T, dtype="bf16")
    q = torch.randn(T, hq * dh, device=dev)
    k = torch.randn(T, hkv * dh, device=dev)
    v = torch.randn(T, hkv * dh, device=dev)
    v[3, 5] = 1e5
    g = torch.ones(dh, device=dev)
    nm.attn_prologue(cache, 0, q, k, v, g, g, 1e-6, 1e6, 1, 1, gated=False)
    with pytest.raises(_lib.ValueOverflow):
        nm.device_status(0)
    nm.device_status(0)
