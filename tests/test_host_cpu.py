"""Host-side bookkeeping on the CPU: input normalization, per-call indices, validation
order and cache growth policy, checked bit-exactly against the oracle's restatement of
reference/qwen38_inference.py (REF:4821-4841, 4966-5044)."""
import math

import numpy as np
import pytest
import torch

from oracle.model import metadata as oracle_metadata, token_batch as oracle_token_batch
from qwen38_inference_b200 import model as M
from qwen38_inference_b200.config import mini

FORMS = [
    [1, 2, 3],
    [[1, 2], [3]],
    ((4, 5), (6,)),
    torch.tensor([1, 2, 3], dtype=torch.int32),
    torch.tensor([[1, 2], [3, 4]], dtype=torch.int64),
    torch.arange(8, dtype=torch.int64).view(2, 4)[:, ::2],
    [torch.tensor([7, 8]), torch.tensor([9], dtype=torch.int32)],
]
BAD = [[], [[]], [[1], []], torch.zeros(2, 2, 2, dtype=torch.int64), torch.zeros(3), [1.0, 2.0], [[1, 2.5]],
       "abc", [torch.zeros(2, 2, dtype=torch.int64)], [True, 2], [[1, np.int64(3)]], [[4], [5, False]]]


@pytest.mark.parametrize("x", FORMS)
def test_token_batch_matches_reference_rules(x):
    assert M._token_batch(x) == oracle_token_batch(x)


@pytest.mark.parametrize("x", BAD)
def test_token_batch_rejects(x):
    with pytest.raises(ValueError):
        oracle_token_batch(x)
    with pytest.raises(ValueError):
        M._token_batch(x)


@pytest.mark.parametrize("case", [
    dict(lengths=[0, 0, 0], slots=[0, 1, 2], lens=[5, 64, 130], cap=192),
    dict(lengths=[63, 0, 128, 7], slots=[2, 0, 3], lens=[1, 1, 1], cap=256),
    dict(lengths=[1023, 4095, 2047], slots=[1, 2, 0], lens=[1, 1, 1], cap=4096),
    dict(lengths=[10, 20], slots=[1], lens=[300], cap=384),
])
def test_metadata_bit_exact(case):
    lengths, slots, lens, cap = case["lengths"], case["slots"], case["lens"], case["cap"]
    ref = oracle_metadata(lengths, cap, slots, lens)
    packed, offs, T = M.build_metadata(slots, ref["prefixes"], lens, cap)
    get = lambda k: packed[offs[k][0]:offs[k][0] + offs[k][1]].tolist()
    assert T == sum(lens)
    assert get("cu") == ref["cu"]
    assert get("positions") == ref["positions"]
    assert get("locations") == ref["locations"]
    assert get("slots") == slots
    assert get("has_initial") == [int(h) for h in ref["has_initial"]]
    assert get("seq_len") == ref["lengths"]
    assert get("last_rows") == [e - 1 for e in ref["cu"][1:]]
    # kv_base is where the reference page table points: page j of request i starts at row
    # 64 * page_table[i][j] = kv_base[i] + 64 j for every live page
    kvb = get("kv_base")
    for i, row in enumerate(ref["page_table"]):
        live = math.ceil(ref["lengths"][i] / 64)
        for j, page in enumerate(row):
            if j < live:
                assert page * 64 == kvb[i] + 64 * j
            else:
                assert page == 0
    # attention tiles cover every query of every request exactly once, longest first
    tiles = np.asarray(get("tiles")).reshape(-1, 2)
    cover = set()
    for r, q0 in tiles.tolist():
        for q in range(q0, min(q0 + 128, lens[r])):
            assert (r, q) not in cover
            cover.add((r, q))
    assert cover == {(r, q) for r in range(len(lens)) for q in range(lens[r])}
    work = [ref["prefixes"][r] + q0 for r, q0 in tiles.tolist()]
    assert work == sorted(work, reverse=True)


class _StubEngine:
    """Records calls instead of launching kernels (host-logic tests only)."""

    def __init__(self, vocab):
        self.vocab = vocab
        self.calls = []
        self.next_token = None  # f(last id of a row) = the argmax of its logits; None: all zero

    def forward(self, flat, slots, prefixes, lens, cache, is_decode, all_logits, dev_tokens=None):
        self.calls.append(dict(slots=list(slots), prefixes=list(prefixes), lens=list(lens), is_decode=is_decode,
                               device_tokens=dev_tokens is not None))
        n = sum(lens) if all_logits else len(lens)
        out = torch.zeros(n, self.vocab)
        if self.next_token is not None and not all_logits:
            ids = dev_tokens.tolist() if dev_tokens is not None else flat
            for r, last in enumerate(np.cumsum(lens) - 1):
                out[r, self.next_token(ids[last])] = 1.0
        return out

    def check_device_error(self, block=False):
        self.calls and self.calls[-1].setdefault("checked", True)


def _cpu_kv_grow(src_k, src_v, dst_k, dst_v, lengths, S, old_cap, new_cap):
    dst_k.zero_()
    dst_v.zero_()
    for s, L in enumerate(lengths.tolist()):
        dst_k[64 + s * new_cap:64 + s * new_cap + L] = src_k[64 + s * old_cap:64 + s * old_cap + L]
        dst_v[64 + s * new_cap:64 + s * new_cap + L] = src_v[64 + s * old_cap:64 + s * old_cap + L]


@pytest.fixture
def host_model(monkeypatch):
    cfg = mini(num_layers=4, vocab=64)
    m = object.__new__(M.Qwen38)
    m.cfg, m.config = cfg, cfg.text_config()
    m.device, m.dtype, m.eps = torch.device("cpu"), torch.bfloat16, cfg.rms_norm_eps
    m.max_context, m.layer_types, m.page_size = 1000, cfg.layer_types, 64
    m.eos_token_ids = {cfg.eos_token_id}
    m._engine = _StubEngine(cfg.vocab_size)
    m._arena = M._BufferArena(m.device)
    monkeypatch.setattr(M.ops, "kv_grow", _cpu_kv_grow)
    monkeypatch.setattr(M.ops, "kv_grow_layers", lambda src, dst, lengths, S, old_cap, new_cap: [
        _cpu_kv_grow(sk, sv, dk, dv, lengths, S, old_cap, new_cap) for (sk, sv), (dk, dv) in zip(src, dst)])
    return m


def test_arena_reuses_buffers_of_dead_caches(host_model):
    """A fresh cache gets the (zeroed) buffers of a dead one, growth hands the replaced KV
    pools back, and no buffer is ever owned by two live caches."""
    import gc
    m = host_model
    a = m.new_cache(2, initial_capacity=64)
    ptrs_a = sorted(t.data_ptr() for t in a._arena_box)
    with torch.inference_mode():
        a.recurrent[0].fill_(3.0)
    a.lengths = [10, 0]
    m._reserve(a, 100)  # grow: the 64-capacity pools go back to the arena
    grown = sorted(t.data_ptr() for t in a._arena_box)
    b = m.new_cache(2, initial_capacity=64)  # takes the pools a gave back
    ptrs_b = sorted(t.data_ptr() for t in b._arena_box)
    assert set(ptrs_b) & set(grown) == set()  # a is alive: nothing shared with it
    assert set(ptrs_b) & set(ptrs_a)  # the returned 64-capacity pools are reused
    del a
    gc.collect()
    c = m.new_cache(2, initial_capacity=64)
    assert set(t.data_ptr() for t in c._arena_box) & set(grown)  # a's state buffers came back
    assert float(c.recurrent[0].abs().sum()) == 0.0 and float(c.kv[3][0].abs().sum()) == 0.0
    live = [t.data_ptr() for t in b._arena_box] + [t.data_ptr() for t in c._arena_box]
    assert len(live) == len(set(live))


def test_new_cache_and_growth_policy(host_model):
    m = host_model
    c = m.new_cache(3, initial_capacity=10)
    assert c.capacity == 64 and c.lengths == [0, 0, 0]
    k, _ = c.kv[3]
    assert k.shape[0] == 3 * 64 + 64
    with torch.inference_mode():
        k[64:64 + 5] = 1.0  # slot 0 live rows
        k[64 + 64:64 + 64 + 40] = 2.0  # slot 1 rows, only 3 live
    c.lengths = [5, 3, 0]
    m._reserve(c, 65)  # doubling: max(65, 128) -> 128
    assert c.capacity == 128
    k2, _ = c.kv[3]
    assert k2.shape[0] == 3 * 128 + 64
    assert bool((k2[64:69] == 1).all()) and bool((k2[69:192] == 0).all())
    assert bool((k2[192:195] == 2).all()) and bool((k2[195:320] == 0).all())  # stale rows not copied
    m._reserve(c, 600)  # needed > 2*cap
    assert c.capacity == 640
    m._reserve(c, 1000)
    assert c.capacity == 1024 or c.capacity == math.ceil(min(1000, max(1000, 1280)) / 64) * 64
    with pytest.raises(ValueError):
        m._reserve(c, 1001)


def test_generate_window_matches_stepwise(host_model, monkeypatch):
    """generate's device-token windows (several decode steps between host reads) produce the
    step-by-step loop's tokens (window 1 is REF's loop, REF:5133-5146) through EOS inside a
    window, max_new_tokens and context exhaustion, with a stub whose next token is a fixed
    function of the last one (+2 mod 64: odd EOS ids are never reached from even ids)."""
    m = host_model
    m._engine.next_token = lambda t: (t + 2) % 64

    def run(window, *args, **kw):
        monkeypatch.setattr(M.Qwen38, "GEN_WINDOW", window)
        m._engine.calls.clear()
        try:
            out = m.generate(*args, **kw)
        except RuntimeError as e:
            out = ("RuntimeError", str(e))
        return out, [c["device_tokens"] for c in m._engine.calls]

    cases = [
        # request 0 meets EOS (8 = 2 + 6) at its third token, inside the first window
        (([[2], [10, 4], [20, 20, 20]],), dict(max_new_tokens=11, eos_token_ids=[8])),
        (([[2], [11]],), dict(max_new_tokens=3, eos_token_ids=[1])),
        (([[2, 4]],), dict(max_new_tokens=9, eos_token_ids=[1])),
        # no EOS reachable: runs until the context (1000) is exhausted
        (([[2] * 990, [4] * 3],), dict(eos_token_ids=[1])),
        (([[2] * 990],), dict(eos_token_ids=[1], max_new_tokens=10)),
    ]
    for args, kw in cases:
        want, step_calls = run(1, *args, **kw)
        got, win_calls = run(8, *args, **kw)
        assert got == want, (args, kw)
        assert not any(step_calls)
        assert any(win_calls) or kw.get("max_new_tokens", 2) <= 1
    assert run(8, [[2], [10, 4], [20, 20, 20]], max_new_tokens=11, eos_token_ids=[8])[0][0] == [4, 6, 8]
    assert run(8, [[2] * 990], eos_token_ids=[1])[0] == (
        "RuntimeError", "Request 0 exhausted context without EOS; produced 11 tokens")


def test_forward_step_validation_before_mutation(host_model):
    m = host_model
    c = m.new_cache(2, initial_capacity=64)
    for bad in ([[1, 2], [64]], [[-1], [2]], [[1], [2 ** 70]], [[1], [-2 ** 70]]):
        with pytest.raises(ValueError):
            m.forward_step(bad, c)
    with pytest.raises(ValueError):
        m.forward_step([[1]], c, request_indices=[5])
    with pytest.raises(ValueError):
        m.forward_step([[1], [2]], c, request_indices=[1, 1])
    with pytest.raises(ValueError):
        m.forward_step([[1], [2]], c, request_indices=[0])
    foreign = m.new_cache(2)
    foreign.owner = 0
    with pytest.raises(ValueError):
        m.forward_step([[1], [2]], foreign)
    assert c.lengths == [0, 0] and m._engine.calls == []


def test_decode_rule_and_length_commit(host_model):
    m = host_model
    c = m.new_cache(3, initial_capacity=64)
    out = m.forward_step([[1, 2], [3]], c, request_indices=[2, 0])
    assert out.shape == (2, 64) and c.lengths == [1, 0, 2]
    assert m._engine.calls[-1]["is_decode"] is False
    m.forward_step([[4], [5]], c, request_indices=[0, 2])
    assert m._engine.calls[-1]["is_decode"] is True and c.lengths == [2, 0, 3]
    # a new slot in the call makes it a prefill (REF:5027)
    m.forward_step([[4], [5]], c, request_indices=[1, 2])
    assert m._engine.calls[-1]["is_decode"] is False
    out = m.forward_step([[1, 2, 3], [4]], c, request_indices=[0, 1], return_all_logits=True)
    assert out.shape == (4, 64)
    with pytest.raises(ValueError):
        m.forward_step([[1] * 997], c, request_indices=[2])  # 4 + 997 > max_context 1000
    c.reset([0])
    assert c.lengths[0] == 0


def test_generate_contract(host_model):
    m = host_model
    out = m.generate([1, 2, 3], max_new_tokens=3, eos_token_ids=[63])
    assert isinstance(out, list) and len(out) == 3 and all(type(t) is int for t in out)
    assert m.generate([[1], [2, 3]], max_new_tokens=0) == [[], []]
    with pytest.raises(ValueError):
        m.generate([1], max_new_tokens=-1)
    with pytest.raises(ValueError):
        m.generate([1], prefill_chunk_size=0)
    with pytest.raises(ValueError):
        m.generate([1], eos_token_ids=[64])
    # chunked prefill: each chunk is one forward_step over the requests that still have input
    m._engine.calls.clear()
    m.generate([[1] * 5, [2] * 2], max_new_tokens=1, prefill_chunk_size=2)
    assert [c["slots"] for c in m._engine.calls] == [[0, 1], [0], [0]]
    # the 1-token tail chunk of an already-started request is classified decode (REF:5027)
    assert [c["is_decode"] for c in m._engine.calls] == [False, False, True]
