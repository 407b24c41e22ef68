"""Host logic of head-wise tensor parallelism, on the CPU.

* Sharded geometry of the 27B model at 1/2/4/8 ranks, including KV heads replicated over
  ranks when there are fewer KV heads than ranks.
* The shards compute what the unsharded weights compute (fp32 on the CPU):
  - column-parallel projections give the rank's slice of the full output;
  - row-parallel projections sum to the full output;
  - the vocabulary shards tile the logits.
* The collectives of ``TensorParallel`` on two gloo ranks.
"""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qwen38_inference_b200.config import mini, qwen38_27b, random_weights, tiny
from qwen38_inference_b200.tensor_parallel import ShardSpec, check_shardable, shard_config, shard_tensor

ROOT = Path(__file__).resolve().parents[1]


def test_27b_shard_geometry():
    c = qwen38_27b()
    for world, (nq, nkv, hk, hv, inter) in {1: (24, 4, 16, 48, 17408), 2: (12, 2, 8, 24, 8704),
                                            4: (6, 1, 4, 12, 4352), 8: (3, 1, 2, 6, 2176)}.items():
        lc = shard_config(c, world)
        assert (lc.num_attention_heads, lc.num_key_value_heads, lc.linear_num_key_heads,
                lc.linear_num_value_heads, lc.intermediate_size) == (nq, nkv, hk, hv, inter)
        assert lc.vocab_size == c.vocab_size and lc.hidden_size == c.hidden_size
    # 8 ranks: 3 query heads each; KV head h serves query heads 6h..6h+5, i.e. ranks 2h, 2h+1
    assert [ShardSpec(r, 8, c).kv_head0 for r in range(8)] == [0, 0, 1, 1, 2, 2, 3, 3]
    assert [ShardSpec(r, 4, c).kv_head0 for r in range(4)] == [0, 1, 2, 3]
    for bad in (3, 5, 16):
        with pytest.raises(ValueError):
            check_shardable(c, bad)


def test_per_rank_leading_dimensions_are_16_byte_multiples():
    """Every buffer the engine hands to a kernel as rows of a wider matrix has a row stride
    of a multiple of 8 bf16 elements at 1, 2, 4 and 8 ranks (the conv, GDN and attention
    kernels read column blocks of the projection buffer with 16-byte and TMA loads)."""
    from qwen38_inference_b200.engine import proj_stride
    c = qwen38_27b()
    for world in (1, 2, 4, 8):
        lc = shard_config(c, world)
        stride = proj_stride(lc)
        assert stride % 8 == 0 and stride >= lc.qkv_dim and stride >= lc.qkvz_dim + lc.ba_dim
        for width in (lc.attn_out_dim, lc.gdn_v_dim, lc.intermediate_size, lc.gdn_qk_dim, lc.conv_dim,
                      lc.hidden_size, c.vocab_size // world):
            assert width % 8 == 0, (world, width)
    assert proj_stride(shard_config(c, 8)) == 2064  # 2048 qkvz + 12 ba, rounded up
    assert proj_stride(c) == 16480  # one GPU: unchanged


def _shards(cfg, world, seed=3):
    full = random_weights(cfg, seed, dtype=torch.float32)
    per_rank = [{k: shard_tensor(k, v, ShardSpec(r, world, cfg)) for k, v in full.items()} for r in range(world)]
    # the shard hook of random_weights gives the same slices as slicing afterwards
    hooked = random_weights(cfg, seed, dtype=torch.float32, shard=lambda k, t: shard_tensor(k, t, ShardSpec(1, world, cfg)))
    for k in full:
        assert torch.equal(hooked[k], per_rank[1][k]), k
    return full, per_rank


def _heads(x, head_dim, heads):
    """Columns of the given heads of x [T, n*head_dim]."""
    return torch.cat([x[:, h * head_dim:(h + 1) * head_dim] for h in heads], 1)


@pytest.mark.parametrize("cfg_name,world", [("mini", 2), ("tiny", 2), ("tiny", 4)])
def test_shards_compute_the_unsharded_model(cfg_name, world):
    cfg = {"mini": mini(num_layers=4, vocab=2048), "tiny": tiny()}[cfg_name]
    full, ranks = _shards(cfg, world)
    g = torch.Generator().manual_seed(0)
    T, H = 5, cfg.hidden_size
    x = torch.randn(T, H, generator=g)
    for i, kind in enumerate(cfg.layer_types):
        p = f"layers.{i}."
        # MLP: column-parallel gate/up, row-parallel down
        I = cfg.intermediate_size
        gu = x @ full[p + "gate_up"].T
        act = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
        want = act @ full[p + "down"].T
        got = 0
        for r in range(world):
            gur = x @ ranks[r][p + "gate_up"].T
            Ir = gur.shape[1] // 2
            got = got + (torch.nn.functional.silu(gur[:, :Ir]) * gur[:, Ir:]) @ ranks[r][p + "down"].T
        torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)
        if kind == "full_attention":
            d, nq, nkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
            y = x @ full[p + "qkv"].T
            qg, k, v = y[:, :2 * nq * d], y[:, 2 * nq * d:2 * nq * d + nkv * d], y[:, 2 * nq * d + nkv * d:]
            att = torch.randn(T, nq * d, generator=g)  # stands for the attention output
            want_o = att @ full[p + "out"].T
            got_o = 0
            for r in range(world):
                sp = ShardSpec(r, world, cfg)
                yr = x @ ranks[r][p + "qkv"].T
                qheads = range(r * sp.nq, (r + 1) * sp.nq)
                kvheads = range(sp.kv_head0, sp.kv_head0 + sp.nkv)
                torch.testing.assert_close(yr[:, :2 * sp.nq * d], _heads(qg, 2 * d, qheads))
                torch.testing.assert_close(yr[:, 2 * sp.nq * d:2 * sp.nq * d + sp.nkv * d], _heads(k, d, kvheads))
                torch.testing.assert_close(yr[:, 2 * sp.nq * d + sp.nkv * d:], _heads(v, d, kvheads))
                # every local query head uses a local KV head under the local GQA grouping
                for hl, h in enumerate(qheads):
                    assert h // (nq // nkv) == sp.kv_head0 + hl // (sp.nq // sp.nkv)
                got_o = got_o + _heads(att, d, qheads) @ ranks[r][p + "out"].T
                for n in ("q_norm", "k_norm", "input_norm", "post_norm"):
                    assert torch.equal(ranks[r][p + n], full[p + n])
            torch.testing.assert_close(got_o, want_o, rtol=1e-5, atol=1e-5)
        else:
            dk, dv, Hk, HV = (cfg.linear_key_head_dim, cfg.linear_value_head_dim, cfg.linear_num_key_heads,
                              cfg.linear_num_value_heads)
            y = x @ full[p + "qkvz"].T
            q, k = y[:, :Hk * dk], y[:, Hk * dk:2 * Hk * dk]
            v, z = y[:, 2 * Hk * dk:2 * Hk * dk + HV * dv], y[:, 2 * Hk * dk + HV * dv:]
            ba = x @ full[p + "ba"].T
            o = torch.randn(T, HV * dv, generator=g)  # stands for the gated-norm output
            want_o = o @ full[p + "out"].T
            got_o = 0
            for r in range(world):
                sp = ShardSpec(r, world, cfg)
                yr = x @ ranks[r][p + "qkvz"].T
                kh, vh = range(r * sp.hk, (r + 1) * sp.hk), range(r * sp.hv, (r + 1) * sp.hv)
                exp = torch.cat([_heads(q, dk, kh), _heads(k, dk, kh), _heads(v, dv, vh), _heads(z, dv, vh)], 1)
                torch.testing.assert_close(yr, exp)
                # value head hv uses QK head hv // (HV / Hk), locally as well
                for hl, h in enumerate(vh):
                    assert h // (HV // Hk) == r * sp.hk + hl // (sp.hv // sp.hk)
                bar = x @ ranks[r][p + "ba"].T
                torch.testing.assert_close(bar, torch.cat([ba[:, list(vh)], ba[:, [HV + h for h in vh]]], 1))
                conv_rows = (list(range(r * sp.hk * dk, (r + 1) * sp.hk * dk))
                             + list(range(Hk * dk + r * sp.hk * dk, Hk * dk + (r + 1) * sp.hk * dk))
                             + list(range(2 * Hk * dk + r * sp.hv * dv, 2 * Hk * dk + (r + 1) * sp.hv * dv)))
                assert torch.equal(ranks[r][p + "conv"], full[p + "conv"][conv_rows])
                assert torch.equal(ranks[r][p + "A_log"], full[p + "A_log"][list(vh)])
                assert torch.equal(ranks[r][p + "dt_bias"], full[p + "dt_bias"][list(vh)])
                assert torch.equal(ranks[r][p + "norm"], full[p + "norm"])
                got_o = got_o + _heads(o, dv, vh) @ ranks[r][p + "out"].T
            torch.testing.assert_close(got_o, want_o, rtol=1e-5, atol=1e-5)
    # vocabulary shards tile the lm_head; the embedding is replicated
    assert torch.equal(torch.cat([rk["lm_head"] for rk in ranks], 0), full["lm_head"])
    assert all(torch.equal(rk["embedding"], full["embedding"]) for rk in ranks)


def test_prefill_attention_split_choice():
    from qwen38_inference_b200.ops import prefill_attn_splits
    # a B32 x L1024 prefill fills the SMs with heads x tiles: no split
    assert prefill_attn_splits(24, 256, 1024) == 1
    # short keys: no split whatever the grid
    assert prefill_attn_splits(3, 4, 1024) == 1
    # one 512-token chunk at 128k context: heads x 4 tiles leave SMs idle, so split
    s1, s8 = prefill_attn_splits(24, 4, 131072), prefill_attn_splits(3, 4, 131072)
    assert s1 > 1 and s8 > s1
    assert 24 * 4 * s1 >= 140 and 3 * 4 * s8 >= 140  # about a wave of the 148 SMs or more
    assert (131072 // 64) // s8 >= 8  # at least 8 key blocks per split


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qwen38_inference_b200.tensor_parallel import TensorParallel
        tp = TensorParallel(None, qwen38_27b())
        part = torch.full((3, 4), float(rank + 1))
        tp.all_reduce_(part)
        local = torch.arange(6, dtype=torch.float32).reshape(2, 3) + 100 * rank
        gathered = torch.empty(world * 2, 3)
        tp.all_gather_rows(local, gathered)
        out[rank] = (tp.rank, tp.world, tp.local_cfg.num_attention_heads, part.tolist(), gathered.tolist())
    finally:
        dist.destroy_process_group()


def test_two_rank_collectives():
    world = 2
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank_main, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        rank, w, nq, part, gathered = res[r]
        assert (rank, w, nq) == (r, 2, 12)
        assert part == [[3.0] * 4] * 3  # 1 + 2
        # rank-major: rank 0's rows, then rank 1's
        assert gathered == [[0, 1, 2], [3, 4, 5], [100, 101, 102], [103, 104, 105]]
