"""ViT encoder on the native path (2-D RoPE + paged KV write kernel, bidirectional tcgen05
flash attention, batched over images) against the fp32 torch encoder (per-image SDPA)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("size", [64, 96, 128])
def test_vision_forward_native_matches_fp32(cuda, size):
    from mod_b200.config import get_preset
    from mod_b200.models.backend import TorchBackend, make_backend
    from mod_b200.models.vl import ViTBlock, VisionWeights, preprocess, random_vision_weights, vision_forward
    from mod_b200.ops import check_status

    cfg = get_preset("tiny-vl")
    vc = cfg.vision  # hidden 128, 2 heads: head_dim 64
    vw = random_vision_weights(vc, device=cuda, dtype=torch.bfloat16, seed=3)
    g = torch.Generator().manual_seed(2)
    imgs = torch.rand(3, 3, size, size, generator=g).to(cuda)
    patches = preprocess(imgs, vc, size)
    out = vision_forward(vc, vw, patches.to(torch.bfloat16), make_backend("native"), size)
    torch.cuda.synchronize()
    check_status()

    def f32(v):
        return v.float() if isinstance(v, torch.Tensor) else v

    vw32 = VisionWeights(**{k: (f32(v) if not isinstance(v, list) else
                                [ViTBlock(**{kk: f32(vv) for kk, vv in vars(b).items()}) for b in v])
                            for k, v in vars(vw).items()})
    ref = vision_forward(vc, vw32, patches.float(), TorchBackend(), size)
    scale = ref.abs().max().item()
    err = (out.float() - ref).abs().max().item()
    assert err < 5e-2 * max(1.0, scale), (err, scale)
