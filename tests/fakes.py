"""Small module trees with the attribute layout of the Gemma text decoder, for tests."""
import torch


def fake_model(layers=3, d=64, inter=128, heads=(4, 1, 1), hd=16, ple=32, shared_from=2):
    """A module tree with the attribute names to_npu walks (gemma_npu.py:209-224)."""
    H, KV, _ = heads
    L = torch.nn.Linear
    lm = torch.nn.Module()
    lm.layers = torch.nn.ModuleList()
    for i in range(layers):
        layer = torch.nn.Module()
        a = torch.nn.Module()
        a.is_kv_shared_layer = i >= shared_from
        a.q_proj = L(d, H * hd, bias=False)
        a.k_proj = L(d, KV * hd, bias=False)
        a.v_proj = L(d, KV * hd, bias=False)
        a.o_proj = L(H * hd, d, bias=False)
        mlp = torch.nn.Module()
        mlp.gate_proj = L(d, inter, bias=False)
        mlp.up_proj = L(d, inter, bias=False)
        mlp.down_proj = L(inter, d, bias=False)
        layer.self_attn, layer.mlp = a, mlp
        layer.per_layer_input_gate = L(d, ple, bias=False)
        layer.per_layer_projection = L(ple, d, bias=False)
        lm.layers.append(layer)
    lm.per_layer_model_projection = L(d, layers * ple, bias=False)
    model = torch.nn.Module()
    model.model = torch.nn.Module()
    model.model.language_model = lm
    model.lm_head = L(d, 512, bias=False)
    return model
