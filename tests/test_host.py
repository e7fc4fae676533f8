"""Host-side logic of the B200 linears that needs no GPU: grouping, slicing, sharding,
the request protocol and input validation."""
import argparse
import types

import pytest
import torch

import gemma_npu_b200 as w8
from gemma_npu_b200 import gemm as g8
from gemma_npu_b200.lm_head import shard_rows

from fakes import fake_model


def test_layer_groups_follow_the_reference_grouping():
    m = fake_model()
    groups, keys = g8.layer_groups(m.model.language_model)
    assert len(groups) == 6 * 3 + 1
    assert keys == [["qkv", "o", "gate_up", "down", "ple_gate", "ple_proj"]] * 3
    names = [tuple(n) for _, n, _ in groups]
    assert names[0] == ("q_proj", "k_proj", "v_proj")
    assert names[2] == ("gate_proj", "up_proj")
    assert names[12] == ("q_proj",)  # a KV-shared layer keeps q only (gemma_npu.py:214-216)
    assert names[-1] == ("per_layer_model_projection",)


class FakeGemm:
    def __init__(self, sizes):
        self.sizes, self.pending, self.calls = sizes, None, 0

    def matmul(self, x2d):
        self.calls += 1
        return torch.cat([torch.full((x2d.shape[0], n), float(i)) for i, n in enumerate(self.sizes)], 1)


def test_slice_runs_the_group_once_and_fans_out():
    g = FakeGemm([3, 2, 2])
    parts = [g8.Slice(g, i, 8, n) for i, n in enumerate(g.sizes)]
    x = torch.zeros(2, 5, 8)
    outs = [p(x) for p in parts]
    assert g.calls == 1 and g.pending is None
    for i, (o, n) in enumerate(zip(outs, g.sizes)):
        assert o.shape == (2, 5, n) and bool((o == i).all())
    parts[1](x)  # a later member called with a fresh input recomputes
    assert g.calls == 2


@pytest.mark.parametrize("vocab", [262144, 1001, 7])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_cover_the_vocab(vocab, world):
    seen = []
    for r in range(world):
        r0, r1, per = shard_rows(vocab, world, r)
        want_per = (vocab + world - 1) // world
        want_per = (want_per + 3) // 4 * 4  # shards start on 16-byte boundaries of fp32 logits
        assert 0 <= r1 - r0 <= per and per == want_per and (r0 % 4 == 0 or r0 == vocab)
        seen.extend(range(r0, r1))
    assert seen == list(range(vocab))


def test_gemm_request_protocol():
    calls = []
    fake = types.SimpleNamespace(name="qkv", stage=lambda slot, T: torch.empty(T, 4, dtype=torch.int8),
                                 launch_slot=lambda T, slot: calls.append((T, slot)) or "acc")
    kind, thunk, name = g8.gemm(fake, torch.ones(3, 4, dtype=torch.int8), None, 2)
    assert (kind, name) == ("npu", "qkv") and calls == []
    assert thunk() == "acc" and calls == [(3, 2)]


def test_backend_flag():
    ap = w8.add_backend_argument(argparse.ArgumentParser())
    assert ap.parse_args([]).backend == "b200"
    assert ap.parse_args(["--backend", "cpu-int8"]).backend == "cpu-int8"
    with pytest.raises(ValueError):
        w8.apply_backend(fake_model(), "cpu")


def test_kernels_reject_host_tensors():
    a = torch.zeros(4, 16, dtype=torch.int8)
    with pytest.raises(ValueError, match="CUDA"):
        w8.mm_i8(a, torch.zeros(16, 4, dtype=torch.int8), torch.zeros(4, 4, dtype=torch.int32))
    with pytest.raises(ValueError, match="CUDA"):
        w8.quant_rows(torch.zeros(4, 16))
    with pytest.raises(ValueError, match="CUDA"):
        w8.int8_linear(torch.zeros(1, 16), torch.zeros(4, 16, dtype=torch.int8), torch.zeros(4))


def test_pack_gelu_up_layout():
    """Packed row 256t + j = gate row 128t + j; packed row 256t + 128 + j = up row I + 128t + j."""
    import torch

    inter, k = 384, 16
    w = torch.arange(2 * inter, dtype=torch.int32)[:, None].expand(2 * inter, k).to(torch.int8).contiguous()
    rows = torch.arange(2 * inter, dtype=torch.float32)
    wp, sp = w8.pack_gelu_up(torch.arange(2 * inter)[:, None].expand(2 * inter, k).contiguous(), rows)
    for t in range(inter // 128):
        for j in (0, 5, 127):
            assert sp[256 * t + j].item() == 128 * t + j
            assert sp[256 * t + 128 + j].item() == inter + 128 * t + j
            assert wp[256 * t + 128 + j, 3].item() == inter + 128 * t + j
    assert w.shape == wp.shape


def test_greedy_key_merge_matches_argmax():
    """Sharded greedy decode: per-shard keys merged on the host pick torch.argmax's token
    (largest value, lowest id on ties), for negative, positive and tied logits."""
    from gemma_npu_b200 import kernels, lm_head

    gen = torch.Generator().manual_seed(0)
    for v in (torch.randn(1000, generator=gen), -torch.rand(1000, generator=gen) - 1,
              torch.tensor([1.0, 3.0, 3.0, 2.0, 3.0])):
        shards = torch.tensor_split(torch.arange(v.numel()), 4)
        keys = []
        for idx in shards:
            local = v[idx]
            j = int(local.argmax())
            keys.append(lm_head.merge_key(kernels.monotone_bits(local[j:j + 1])[0], idx[j]))
        tok = lm_head.greedy_from_keys(torch.stack(keys).max())
        assert int(tok) == int(v.argmax())
