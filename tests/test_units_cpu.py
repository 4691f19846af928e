"""Host-side units on CPU: micro-batch split and forward plans, topology role
maps, tag formulas, sampling, tensor comparison, timing JSON round trip and
CLI parsing (the reference's tests/test_pipeline.py, test_correctness.py,
test_input_preparation.py and test_timing_comm.py cover the same ground)."""

import json

import pytest
import torch

from afd_demo_b200.config import PRESETS, ModelConfig, Topology, tiny_qwen3_moe
from afd_demo_b200.parallel.micro_batch import (MicroBatchManager, MicroBatchState,
                                                additive_causal_mask, create_causal_mask,
                                                create_position_ids, make_plan, split_sizes)
from afd_demo_b200.parallel.transport import NcclTransport
from afd_demo_b200.utils import sampling
from afd_demo_b200.utils.timing import (EventType, PipelineTiming, TimingEvent, TimingTracker,
                                        merge_timings)
from afd_demo_b200.utils.validation import compare_tensors, rel_err


# ----------------------------------------------------------------- micro-batches
@pytest.mark.parametrize("batch,n,want", [(8, 2, [4, 4]), (7, 2, [4, 3]), (5, 3, [2, 2, 1]),
                                          (1, 2, [1]), (3, 4, [1, 1, 1]), (0, 2, [])])
def test_split_sizes(batch, n, want):
    assert split_sizes(batch, n) == want
    assert sum(split_sizes(batch, n)) == batch


def test_manager_split_merge_roundtrip():
    ids = torch.arange(7 * 5).view(7, 5)
    mask = torch.ones(7, 5)
    mgr = MicroBatchManager(2)
    mbs = mgr.split_batch(ids, mask)
    assert [mb.batch_size for mb in mbs] == [4, 3]
    assert [mb.batch_offset for mb in mbs] == [0, 4]
    assert all(mb.seq_len == 5 for mb in mbs)
    assert torch.equal(mgr.merge_results([mb.input_ids for mb in mbs]), ids)
    mbs[0].advance_layer()
    assert mbs[0].current_layer == 1
    assert not mgr.all_completed()
    for mb in mbs:
        mb.state = MicroBatchState.COMPLETED
    assert mgr.all_completed()
    mgr.reset()
    assert all(mb.state == MicroBatchState.WAITING and mb.current_layer == 0 for mb in mbs)


def test_positions_and_masks():
    pos = create_position_ids(2, 4, "cpu", start=3)
    assert pos.tolist() == [[3, 4, 5, 6]] * 2
    cm = create_causal_mask(1, 3, "cpu")
    assert cm[0, 0].tolist() == [[1, 0, 0], [1, 1, 0], [1, 1, 1]]
    am = additive_causal_mask(2, 3, 3, "cpu")
    assert am.shape == (2, 1, 3, 3)
    assert am[0, 0, 0, 0] == 0 and am[0, 0, 0, 1] == torch.finfo(torch.float32).min
    dec = additive_causal_mask(2, 1, 9, "cpu")  # decode: all keys visible
    assert torch.all(dec == 0)


@pytest.mark.parametrize("world,batch", [(2, 4), (4, 6), (8, 32), (8, 9)])
def test_forward_plan_covers_batch(world, batch):
    topo = Topology.for_world(world)
    plan = make_plan(topo, batch, 2, q_len=3)
    seen = []
    for a, r in enumerate(plan.attn_batches):
        slots = plan.slots_of(a)
        assert sum(s.batch_size for s in slots) == len(r)
        off = 0
        for s in slots:
            assert s.batch_offset == off
            off += s.batch_size
            assert s.tokens == s.batch_size * 3
        seen.extend(r)
    assert seen == list(range(batch))
    for m, fs in enumerate(plan.ffn_slots):
        assert fs.seg_tokens == [plan.attn_slots[a][m].tokens for a in range(topo.n_attn)]
        assert fs.seg_offsets[0] == 0
        assert fs.tokens == sum(fs.seg_tokens)


def test_forward_plan_rejects_empty_rank():
    with pytest.raises(ValueError):
        make_plan(Topology.for_world(8), 3, 2, 1)


# ----------------------------------------------------------------- topology
def test_topology_role_maps():
    t1 = Topology.for_world(1)
    assert t1.colocated and t1.role_of(0) == "both" and t1.tag() == "1G"
    t2 = Topology.for_world(2)
    assert [t2.role_of(r) for r in range(2)] == ["attention", "ffn"]
    t8 = Topology.for_world(8)
    assert t8.attn_ranks() == [0, 1, 2, 3] and t8.ffn_ranks() == [4, 5, 6, 7]
    assert t8.tag() == "4A4F"
    assert [t8.experts_of(i, 128) for i in range(4)] == [range(0, 32), range(32, 64),
                                                           range(64, 96), range(96, 128)]
    assert Topology.for_world(6, n_attn=2).tag() == "2A4F"
    with pytest.raises(ValueError):
        Topology.for_world(4, n_attn=4)
    with pytest.raises(ValueError):
        Topology.for_world(8, n_attn=5).experts_of(0, 128)  # 128 over 3 FFN ranks


def test_batch_slices_partition():
    t = Topology.for_world(8)
    for batch in (4, 5, 33, 256):
        parts = [t.batch_slice(a, batch) for a in range(4)]
        assert [i for p in parts for i in p] == list(range(batch))
        assert max(map(len, parts)) - min(map(len, parts)) <= 1


# ----------------------------------------------------------------- config
def test_config_hf_roundtrip(tmp_path):
    cfg = PRESETS["qwen3-30b-a3b"]()
    assert (cfg.hidden_size, cfg.num_hidden_layers, cfg.num_experts) == (2048, 48, 128)
    assert (cfg.q_size, cfg.kv_size, cfg.gqa_group) == (4096, 512, 8)
    cfg.save(str(tmp_path))
    d = json.load(open(tmp_path / "config.json"))
    assert d["model_type"] == "qwen3_moe"
    back = ModelConfig.from_pretrained(str(tmp_path))
    assert back.to_hf_dict() == cfg.to_hf_dict()


def test_config_reads_transformers5_names():
    d = PRESETS["qwen3-30b-a3b"]().to_hf_dict()
    d.pop("num_experts")
    d.pop("rope_theta", None)
    d["num_local_experts"] = 64
    d["rope_parameters"] = {"rope_type": "default", "rope_theta": 5e5}
    cfg = ModelConfig.from_dict(d)
    assert cfg.num_experts == 64 and cfg.rope_theta == 5e5


def test_key_ranges_from_mask():
    from afd_demo_b200.parallel.micro_batch import key_ranges_from_mask
    assert key_ranges_from_mask(None) is None
    assert key_ranges_from_mask(torch.ones(3, 5, dtype=torch.long)) is None
    m = torch.tensor([[1, 1, 1, 0, 0], [0, 0, 1, 1, 1], [1, 1, 1, 1, 1]])
    lo, hi = key_ranges_from_mask(m)
    assert lo.tolist() == [0, 2, 0] and hi.tolist() == [3, 5, 5] and lo.dtype == torch.int32
    with pytest.raises(ValueError):
        key_ranges_from_mask(torch.tensor([[1, 0, 1, 1]]))
    with pytest.raises(ValueError):
        key_ranges_from_mask(torch.tensor([[0, 0, 0], [1, 1, 1]]))


def test_sparse_layer_rule():
    cfg = tiny_qwen3_moe()
    cfg.mlp_only_layers = [1]
    assert cfg.is_sparse_layer(0) and not cfg.is_sparse_layer(1)
    cfg.mlp_only_layers = []
    cfg.decoder_sparse_step = 2
    assert [cfg.is_sparse_layer(l) for l in range(4)] == [False, True, False, True]


# ----------------------------------------------------------------- tags
def test_decode_tags_unique_and_ordered():
    L, nmb = 48, 2
    tags = [NcclTransport.tag(l, m, nmb, d) for l in range(L) for m in range(nmb)
            for d in ("a2f", "f2a")]
    assert len(set(tags)) == len(tags)
    assert tags == sorted(tags)
    assert NcclTransport.tag(0, 0, 2, "a2f") == 10000


# ----------------------------------------------------------------- sampling
def test_top_k_and_top_p_filters():
    logits = torch.tensor([[1.0, 3.0, 2.0, 0.0]])
    k = sampling.top_k_filtering(logits, 2)
    assert torch.isinf(k[0, 0]) and torch.isinf(k[0, 3]) and k[0, 1] == 3.0
    p = sampling.top_p_filtering(torch.log(torch.tensor([[0.6, 0.3, 0.05, 0.05]])), 0.8)
    assert torch.isfinite(p[0, :2]).all() and torch.isinf(p[0, 2:]).all()


def test_greedy_and_seeded_sampling():
    logits = torch.randn(4, 50, generator=torch.Generator().manual_seed(0))
    g = sampling.sample_next_token(logits, do_sample=False)
    assert g.shape == (4, 1) and torch.equal(g.view(-1), logits.argmax(-1))
    a = sampling.sample_next_token(logits, 0.7, 10, 0.9, True,
                                   generator=torch.Generator().manual_seed(1))
    b = sampling.sample_next_token(logits, 0.7, 10, 0.9, True,
                                   generator=torch.Generator().manual_seed(1))
    assert torch.equal(a, b)
    top10 = logits.topk(10, -1).indices
    assert all(int(a[i]) in top10[i].tolist() for i in range(4))


def test_repetition_penalty_and_stopping():
    logits = torch.tensor([[2.0, -2.0, 1.0]])
    out = sampling.repetition_penalty(logits, torch.tensor([[0, 1]]), 2.0)
    assert out.tolist() == [[1.0, -4.0, 1.0]]
    stop = sampling.StoppingCriteria(max_length=10, eos_token_id=7)
    ids = torch.zeros(2, 3, dtype=torch.long)
    assert not stop(ids, torch.tensor([7, 1]))
    assert stop(ids, torch.tensor([0, 7]))
    assert sampling.StoppingCriteria(3)(ids, torch.tensor([0, 0]))


# ----------------------------------------------------------------- validation
def test_compare_tensors():
    a = torch.randn(16, 16)
    ok = compare_tensors(a, a.clone())
    assert ok["match"] if isinstance(ok, dict) else ok[0]
    bad = compare_tensors(a, a + 1.0)
    assert not (bad["match"] if isinstance(bad, dict) else bad[0])
    assert rel_err(a, a) == 0.0


# ----------------------------------------------------------------- timing schema
def _timing():
    pt = PipelineTiming(node="attention", num_layers=2, num_micro_batches=2, total_time_ms=10.0,
                        comm_timing_mode="completion", decode_tpot_ms=1.5, gpus=2,
                        topology="1A1F")
    pt.add_event(TimingEvent("attn_compute", 0, 0, 0.0, 0.002, "attention"))
    pt.add_event(TimingEvent("send_transfer", 0, 0, 0.002, 0.003, "attention", 4096,
                             "future"))
    pt.add_event(TimingEvent("recv_wait", 0, 1, 0.003, 0.004, "attention"))
    pt.add_event(TimingEvent("moe_router", 0, 1, 0.003, 0.0035, "attention"))
    return pt


def test_timing_json_roundtrip(tmp_path):
    pt = _timing()
    d = pt.to_dict()
    for key in ("node", "num_layers", "num_micro_batches", "total_time_ms", "comm_timing_mode",
                "total_compute_ms", "total_recv_wait_ms", "total_moe_router_ms",
                "total_moe_experts_ms", "total_moe_shared_or_dense_ms", "compute_ratio",
                "events"):
        assert key in d
    e = d["events"][1]
    assert set(e) == {"type", "layer", "mb", "start", "end", "duration_ms", "node",
                      "tensor_bytes", "tensor_mib", "completion_source"}
    assert e["tensor_mib"] == 4096 / 2**20
    assert abs(d["total_compute_ms"] - 2.0) < 1e-9
    assert abs(d["total_recv_wait_ms"] - 1.0) < 1e-9
    path = tmp_path / "t.json"
    pt.save(str(path))
    back = PipelineTiming.from_dict(json.load(open(path)))
    assert back.to_dict() == d
    assert "compute" in back.summary()


def test_event_type_values():
    assert [e.value for e in EventType] == [
        "attn_compute", "ffn_compute", "moe_router", "moe_experts", "moe_shared_or_dense",
        "send_start", "send_transfer", "recv_post", "recv_wait"]


class _NoFuture:
    """A comm handle whose future is unavailable (gloo / old NCCL Work)."""

    def get_future(self):
        raise RuntimeError("no future")

    def wait(self):
        return True


@pytest.mark.parametrize("mode", ["enqueue", "completion"])
def test_tracker_send_recording(mode):
    tr = TimingTracker("attention", 2, 2, mode="sync", comm_timing_mode=mode)
    tr.mark_start(EventType.ATTN_COMPUTE, 0, 0)
    tr.mark_end(EventType.ATTN_COMPUTE, 0, 0)
    h = _NoFuture()
    import time

    t0 = time.perf_counter()
    tr.record_send(h, 0, 0, t0, tensor=torch.zeros(8, 4))
    tr.observe_send_completion(h)
    pt = tr.finish()
    types = [e.event_type for e in pt.events]
    assert "attn_compute" in types and "send_transfer" in types
    send = [e for e in pt.events if e.event_type == "send_transfer"][0]
    assert send.tensor_bytes == 8 * 4 * 4
    assert send.end_time >= send.start_time
    assert pt.comm_timing_mode == mode


def test_merge_timings():
    a = _timing()
    f = PipelineTiming(node="ffn", num_layers=2, num_micro_batches=2, total_time_ms=9.0)
    f.add_event(TimingEvent("ffn_compute", 0, 0, 0.001, 0.002, "ffn"))
    m = merge_timings(a, f)
    assert isinstance(m, dict)
    assert json.loads(json.dumps(m)) == m


# ----------------------------------------------------------------- CLI
def test_cli_reference_flags():
    from afd_demo_b200.main import get_effective_prefill_seq_len, parse_args

    a = parse_args(["--batch-size", "8", "--prefill-seq-len", "128", "--no-dbo", "--crosslayer",
                    "--max-new-tokens", "20", "--greedy", "--timing", "--warmup-p2p",
                    "--comm-timing-mode", "completion", "--no-generate",
                    "--timing-suffix", "x", "--verbose"])
    assert a.batch_size == 8 and a.no_dbo and a.crosslayer and a.greedy and a.timing
    assert a.max_new_tokens == 20 and a.comm_timing_mode == "completion" and a.no_generate
    assert get_effective_prefill_seq_len(None, 128) == 128
    assert get_effective_prefill_seq_len(64, 128) == 64
    b = parse_args([])
    assert (b.batch_size, b.max_seq_len, b.num_micro_batches, b.dtype) == (2, 128, 2,
                                                                           "bfloat16")


class _FakeTokenizer:
    pad_token_id = 0
    eos_token_id = 1
    pad_token = "<pad>"

    def __call__(self, prompts, return_tensors="pt", padding=True, truncation=False,
                 max_length=None):
        toks = [[2 + (ord(c) % 50) for c in p] for p in prompts]
        if padding == "max_length":
            toks = [t[:max_length] + [0] * max(0, max_length - len(t)) for t in toks]
        else:
            n = max(map(len, toks))
            toks = [t + [0] * (n - len(t)) for t in toks]
        ids = torch.tensor(toks)
        return {"input_ids": ids, "attention_mask": (ids != 0).long()}


def test_prompt_padding_fixed_and_dynamic():
    from afd_demo_b200.main import tokenize_batch_prompts

    tok = _FakeTokenizer()
    fixed, n = tokenize_batch_prompts(tok, ["abc"] * 3, 8, 128)
    assert fixed["input_ids"].shape == (3, 8) and n == 8
    dyn, _ = tokenize_batch_prompts(tok, ["abcd"] * 2, None, 128)
    assert dyn["input_ids"].shape == (2, 4)


def test_yaml_run_config(tmp_path):
    from afd_demo_b200.main import parse_args

    a = parse_args(["--config", "afd_demo_b200/configs/qwen3_30b.yaml", "--batch-size", "8"])
    assert a.batch_size == 8  # command line wins
    assert a.prefill_seq_len == 256 and a.crosslayer and a.cuda_graph and a.greedy
    bad = tmp_path / "bad.yaml"
    bad.write_text("pipeline:\n  not_a_flag: 1\n")
    with pytest.raises(ValueError):
        parse_args(["--config", str(bad)])


def test_tracker_track_context_and_layer_timing():
    from afd_demo_b200.utils.timing import EventType, LayerTiming, TimingTracker
    tr = TimingTracker("attention", 2, 2, mode="sync")
    with tr.track(EventType.ATTN_COMPUTE, 1, 0):
        pass
    pt = tr.finish()
    ev = pt.to_dict()["events"]
    assert [(e["type"], e["layer"], e["mb"]) for e in ev] == [("attn_compute", 1, 0)]
    assert ev[0]["end"] >= ev[0]["start"] >= 0.0
    lt = LayerTiming(3)
    lt.attn_compute.append(1.5)
    assert lt.layer_idx == 3 and lt.ffn_compute == []


def test_every_switch_is_documented():
    """Each AFD_* environment variable the code reads has a README line."""
    import re
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    names = set()
    for p in list((root / "afd_demo_b200").rglob("*.py")) + [root / "bench.py"]:
        names |= set(re.findall(r'environ(?:\.get)?\(?\[?"(AFD_[A-Z0-9_]+)"', p.read_text()))
    for p in (root / "csrc").glob("*"):
        names |= set(re.findall(r'getenv\("(AFD_[A-Z0-9_]+)"', p.read_text()))
    readme = (root / "README.md").read_text()
    assert names and not [n for n in sorted(names) if n not in readme]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_region_addresses_disjoint(world):
    """Address arithmetic of the fused transport's peer regions: every flag
    and data slot of every (micro-batch, peer) lies inside its region, flags
    precede data, slots never overlap, and each attention rank's rows land in
    its own segment of the FFN slot."""
    from afd_demo_b200.config import Topology
    from afd_demo_b200.parallel.micro_batch import make_plan
    from afd_demo_b200.parallel.transport import PeerTransport

    topo = Topology.for_world(world)
    n_attn, n_ffn, H, esz, nmb = len(topo.attn_ranks()), len(topo.ffn_ranks()), 64, 2, 2
    B, S = 8 * n_attn, 5
    plan = make_plan(topo, B, nmb, S)
    Tall = max(s.tokens for s in plan.ffn_slots)
    Ta = max(s.tokens for row in plan.attn_slots for s in row)
    ffn_l, attn_l = PeerTransport.make_layouts(n_attn, n_ffn, nmb, Ta, Tall, H, esz)
    t = PeerTransport.__new__(PeerTransport)
    t.n_attn, t.n_ffn, t.H, t.ffn_layout, t.attn_layout = n_attn, n_ffn, H, ffn_l, attn_l
    base = 1 << 40
    spans = []
    for m in range(nmb):
        for a in range(n_attn):
            f = t._ffn_flag(base, m, a)
            assert base <= f < base + ffn_l.data_offset
            spans.append((f, f + 4))
        lo = t._ffn_data(base, m)
        seg = plan.ffn_slots[m].seg_offsets
        for a in range(n_attn):
            r0 = seg[a]
            r1 = seg[a + 1] if a + 1 < n_attn else plan.ffn_slots[m].tokens
            spans.append((lo + r0 * H * esz, lo + r1 * H * esz))
        assert lo + plan.ffn_slots[m].tokens * H * esz <= base + ffn_l.total
    for m in range(nmb):
        for f in range(n_ffn):
            fl = t._attn_flag(base + (1 << 36), m, f)
            assert base + (1 << 36) <= fl < base + (1 << 36) + attn_l.data_offset
            d = t._attn_data(base + (1 << 36), m, f)
            assert d + Ta * H * esz <= base + (1 << 36) + attn_l.total
            spans.append((fl, fl + 4))
            spans.append((d, d + Ta * H * esz))
    spans = [s for s in spans if s[1] > s[0]]
    spans.sort()
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 <= b0, "overlapping peer-region spans"
