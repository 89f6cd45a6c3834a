"""snapmind_rope_qk against the reference RoPE formula run by torch on the same
device (rotate-half, snapmind/layers/positional/rope.py:47-61): bit-identical
for fp32, bf16 and f16, strided q/k views, positions given or implied."""
import pytest
import torch

from llama_harness import Rope

pytestmark = pytest.mark.gpu


def _torch_rope(x, cos, sin):
    h = x.shape[-1] // 2
    rot = torch.cat((-x[..., h:], x[..., :h]), dim=-1)
    return x * cos + rot * sin


def _run(q, k, cos_t, sin_t, positions, err):
    from snapmind_b200 import _lib

    rc = _lib.load().snapmind_rope_qk(
        q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), q.shape[1],
        k.data_ptr(), k.stride(0), k.stride(1), k.stride(2), k.shape[1],
        _lib.dtype_code(q.dtype), q.shape[0], q.shape[2], q.shape[3], cos_t.data_ptr(), sin_t.data_ptr(),
        cos_t.shape[0], None if positions is None else positions.data_ptr(), 0, err.data_ptr(), _lib.stream_handle(),
    )  # fmt: skip
    _lib.check(rc, "rope")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n_tok,given", [(1, True), (37, False), (37, True)])
def test_rope_kernel_bit_exact(cuda_device, dtype, n_tok, given):
    B, Hq, H, D = 2, 8, 2, 64
    rope = Rope(D, 512, 10000.0).to(cuda_device)
    g = torch.Generator(device="cpu").manual_seed(n_tok)
    # projections laid out as the attention layers make them: (B, T, H, D) viewed as (B, H, T, D)
    q = torch.randn(B, n_tok, Hq, D, generator=g).to(cuda_device, dtype).transpose(1, 2)
    k = torch.randn(B, n_tok, H, D, generator=g).to(cuda_device, dtype).transpose(1, 2)
    pos = (torch.randperm(500, generator=g)[:n_tok] + 3).to(cuda_device) if given else None
    if pos is None:
        cos = rope.cos_cached[:n_tok][None, None].to(dtype)
        sin = rope.sin_cached[:n_tok][None, None].to(dtype)
    else:
        cos = rope.cos_cached[pos].to(dtype)[None, None]
        sin = rope.sin_cached[pos].to(dtype)[None, None]
    want_q, want_k = _torch_rope(q, cos, sin), _torch_rope(k, cos, sin)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _run(q, k, rope.cos_cached, rope.sin_cached, pos, err)
    assert torch.equal(q, want_q) and torch.equal(k, want_k)
    assert int(err.item()) == 0


def test_rope_position_out_of_range_is_flagged(cuda_device):
    from snapmind_b200 import _lib

    rope = Rope(32, 16, 10000.0).to(cuda_device)
    q = torch.randn(1, 2, 3, 32, device=cuda_device)
    k = torch.randn(1, 1, 3, 32, device=cuda_device)
    q0, k0 = q.clone(), k.clone()
    pos = torch.tensor([1, 16, 2], device=cuda_device)  # 16 is past the 16-row tables
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _run(q, k, rope.cos_cached, rope.sin_cached, pos, err)
    assert int(err.item()) & _lib.DEVERR_POSITION
    assert torch.equal(q[:, :, 1], q0[:, :, 1]) and torch.equal(k[:, :, 1], k0[:, :, 1])
    assert not torch.equal(q[:, :, 0], q0[:, :, 0])


@torch.no_grad()
def test_gqa_paged_fused_rope_equals_module_rope(cuda_device):
    """The plugin with the fused kernel and with the PE module's own apply_to_qk
    (a PE without the rotate-half marker) give identical outputs and caches."""
    from snapmind_b200 import ATTENTION, PagedKVCache

    class PlainRope(torch.nn.Module):  # same math, no _rotate_half marker: not fused
        def __init__(self, inner):
            super().__init__()
            self.inner = inner

        def apply_to_qk(self, q, k, position_ids=None):
            return self.inner.apply_to_qk(q, k, position_ids)

    rope = Rope(32, 256, 10000.0).to(cuda_device)
    torch.manual_seed(0)
    fused = ATTENTION.create("gqa_paged", d_model=256, n_heads=8, n_kv_heads=2, pe=rope).to(cuda_device)
    plain = ATTENTION.create("gqa_paged", d_model=256, n_heads=8, n_kv_heads=2, pe=PlainRope(rope)).to(cuda_device)
    plain.load_state_dict(fused.state_dict(), strict=False)
    caches = [PagedKVCache(256, 1, 2, 32), PagedKVCache(256, 1, 2, 32)]
    x = torch.randn(1, 20, 256, device=cuda_device)
    mask = torch.triu(torch.full((20, 20), float("-inf")), diagonal=1).to(cuda_device)
    a, _ = fused(x, kv_cache=caches[0].layer_dicts()[0], mask=mask)
    b, _ = plain(x, kv_cache=caches[1].layer_dicts()[0], mask=mask)
    assert torch.equal(a, b)
    for step in range(3):
        x = torch.randn(1, 1, 256, device=cuda_device)
        p = torch.tensor([20 + step], device=cuda_device)
        a, _ = fused(x, kv_cache=caches[0].layer_dicts()[0], position_ids=p)
        b, _ = plain(x, kv_cache=caches[1].layer_dicts()[0], position_ids=p)
        assert torch.equal(a, b)
    assert torch.equal(caches[0].fetch(0)[0], caches[1].fetch(0)[0])
