"""CPU checks of the config-4 hybrid model's structure (meta device: nothing
is allocated and no kernel runs)."""

import torch


def test_config4_shape_and_names(gdn2):
    from gdn2_b200 import model as m
    with torch.device("meta"):
        net = m.GPT(m.HybridConfig())
    assert m.num_parameters(net) == 1_326_894_784  # ~1.3B
    kinds = [blk.use_gdn2 for blk in net.transformer.h]
    assert len(kinds) == 24 and kinds == [i % 2 == 0 for i in range(24)]
    names = {n for n, _ in net.named_parameters()}
    # the reference's names (lit_gpt/model.py) for a GDN2 block, an attention block and the ends
    for n in ("lm_head.weight", "transformer.wte.weight", "transformer.ln_f.weight",
              "transformer.h.0.norm_1.weight", "transformer.h.0.attn.q_proj.weight",
              "transformer.h.0.attn.o_norm.weight", "transformer.h.0.mlp.swiglu.w3.weight",
              "transformer.h.1.attn.attn.weight", "transformer.h.1.attn.proj.weight",
              "transformer.h.1.norm_2.weight"):
        assert n in names, n
    assert net.lm_head.weight.shape == (32000, 2048)
