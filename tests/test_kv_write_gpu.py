"""Paged KV-cache write (vLLM reshape_and_cache_flash contract) on the B200:
bit-exact against torch's (x.float() / scale).to(float8_e4m3fn) for in-range
values, saturation to +-448 beyond, negative slots skipped."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(T, hkv=8, d=128, pblk=16, nb=64, seed=0, dev="cuda"):
    g = torch.Generator().manual_seed(seed)
    key = torch.randn(T, hkv, d, generator=g).to(torch.bfloat16)
    value = torch.randn(T, hkv, d, generator=g).to(torch.bfloat16)
    slots = torch.randperm(nb * pblk, generator=g)[:T].to(torch.int64)
    return key, value, slots


@pytest.mark.parametrize("T", [1, 7, 100, 1000])
def test_fp8_write_bit_exact(cuda, T):
    import kv_cache
    nb, pblk, hkv, d = 64, 16, 8, 128
    key, value, slots = _setup(T, hkv, d, pblk, nb)
    ks = key.float().abs().max().item() / 448.0
    vs = value.float().abs().max().item() / 448.0
    kc = torch.zeros(nb, pblk, hkv, d, dtype=torch.uint8, device=cuda).view(torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    kv_cache.reshape_and_cache_flash(key.to(cuda), value.to(cuda), kc, vc, slots.to(cuda), "fp8",
                                     torch.tensor([ks], device=cuda), torch.tensor([vs], device=cuda))
    want_k = (key.float() / torch.tensor(ks, dtype=torch.float32)).to(torch.float8_e4m3fn)
    want_v = (value.float() / torch.tensor(vs, dtype=torch.float32)).to(torch.float8_e4m3fn)
    got_k = kc.view(nb * pblk, hkv, d)[slots.to(cuda)].cpu()
    got_v = vc.view(nb * pblk, hkv, d)[slots.to(cuda)].cpu()
    assert torch.equal(got_k.view(torch.uint8), want_k.view(torch.uint8))
    assert torch.equal(got_v.view(torch.uint8), want_v.view(torch.uint8))
    # untouched slots stay zero
    mask = torch.ones(nb * pblk, dtype=torch.bool)
    mask[slots] = False
    assert torch.all(kc.view(nb * pblk, hkv, d).view(torch.uint8)[mask.to(cuda)] == 0)


def test_saturation_and_padding_slots(cuda):
    import kv_cache
    key, value, slots = _setup(16, seed=1)
    key[0, 0, 0] = 1000.0
    key[0, 0, 1] = -1000.0
    slots[3] = -1
    kc = torch.zeros(64, 16, 8, 128, dtype=torch.uint8, device=cuda).view(torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    kv_cache.reshape_and_cache_flash(key.to(cuda), value.to(cuda), kc, vc, slots.to(cuda), "fp8", 1.0, 1.0)
    flat = kc.view(-1, 8, 128).float().cpu()
    assert flat[slots[0], 0, 0] == 448.0 and flat[slots[0], 0, 1] == -448.0
    written = torch.zeros(64 * 16, dtype=torch.bool)
    written[slots[slots >= 0]] = True
    assert torch.all(flat[~written] == 0)


def test_bf16_cache_copy_and_vllm_layout(cuda):
    import kv_cache
    key, value, slots = _setup(50, seed=2)
    kv = torch.zeros(64, 2, 16, 8, 128, dtype=torch.bfloat16, device=cuda)
    kc, vc = kv.unbind(1)
    kv_cache.reshape_and_cache_flash(key.to(cuda), value.to(cuda), kc, vc, slots.to(cuda), "auto", 1.0, 1.0)
    assert torch.equal(kc.reshape(-1, 8, 128)[slots.to(cuda)].cpu(), key)
    assert torch.equal(vc.reshape(-1, 8, 128)[slots.to(cuda)].cpu(), value)
