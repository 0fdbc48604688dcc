"""Quantise-on-load into the stacked layout (mv_quantize_into_stack behind mingmoe.loader's hooks, the
counterpart of ming-voice engine.py:126-147 driven by direct_load.py's loader threads): the int8 rows and scales
written into every slot are bit-exact with the oracle quantiser (fused_moe.py:199-204) of each checkpoint matrix,
for sources on the GPU, in pinned host memory and in pageable host memory, from four threads on four streams."""
import pytest
import torch

from mingmoe import loader
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("scale_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("where", ["cuda", "pinned", "pageable"])
def test_quantise_on_load_into_stacks(cuda, scale_dtype, where):
    E, I, H = 6, 128, 256
    g = torch.Generator().manual_seed(11)
    ckpt = {}
    for layer in range(2):
        for e in range(E):
            for nm, shape in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
                t = (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)
                if where == "cuda":
                    t = t.to(cuda)
                elif where == "pinned":
                    t = t.pin_memory()
                ckpt[f"model.layers.{layer}.mlp.experts.{e}.{nm}.weight"] = t
    stacks = {f"model.layers.{layer}.mlp": (*loader.int8_stacks(E + 1, I, H, cuda, scale_dtype), E)
              for layer in range(2)}
    hooks = loader.int8_expert_loaders(stacks)
    assert set(ckpt) <= set(hooks)
    done = loader.run_hooks(ckpt, hooks, cuda, workers=4)
    assert sorted(done) == sorted(ckpt)
    torch.cuda.synchronize()
    for name, (q_gu, s_gu, q_d, s_d, _) in stacks.items():
        for e in range(E):
            src = [ckpt[f"{name}.experts.{e}.{nm}.weight"].cpu() for nm in ("gate_proj", "up_proj", "down_proj")]
            qg, sg = O.quantize_rows_int8(torch.cat(src[:2]), scale_dtype)
            qd, sd = O.quantize_rows_int8(src[2], scale_dtype)
            assert torch.equal(q_gu[e].cpu(), qg) and torch.equal(s_gu[e].cpu(), sg)
            assert torch.equal(q_d[e].cpu(), qd) and torch.equal(s_d[e].cpu(), sd)


def test_quantise_into_stack_baseline_dims_and_bounds(cuda):
    E1, I, H = 66, 1408, 2048
    q_gu, s_gu, q_d, s_d = loader.int8_stacks(E1, I, H, cuda, torch.bfloat16)
    w = (torch.randn(I, H, generator=torch.Generator().manual_seed(3)) * 0.02).to(torch.bfloat16)
    loader.quantize_into(q_gu, s_gu, 65, I, w.to(cuda))
    torch.cuda.synchronize()
    q, s = O.quantize_rows_int8(w, torch.bfloat16)
    assert torch.equal(q_gu[65, I:].cpu(), q) and torch.equal(s_gu[65, I:].cpu(), s)
    with pytest.raises(RuntimeError, match="outside"):
        loader.quantize_into(q_gu, s_gu, 66, 0, w.to(cuda))
    with pytest.raises(RuntimeError, match="outside"):
        loader.quantize_into(q_gu, s_gu, 0, I + 1, w.to(cuda))
