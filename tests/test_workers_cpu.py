"""The reference's worker constructors (``AttentionWorker.from_pretrained``,
``FFNWorker.from_pretrained``) on CPU: each reads only its role's tensors of a
checkpoint (an expert slice for the FFN), and a preset name gives random
weights of the preset's shape."""

import torch

from afd_demo_b200.config import tiny_qwen3_moe
from afd_demo_b200.models.attention import AttentionWorker
from afd_demo_b200.models.ffn import FFNWorker
from afd_demo_b200.models.weights import (random_attention_weights, random_ffn_weights,
                                          save_checkpoint)


def test_workers_from_a_checkpoint(tmp_path):
    cfg = tiny_qwen3_moe()
    aw0 = random_attention_weights(cfg, 0, "cpu", torch.float32)
    fw0 = random_ffn_weights(cfg, None, 0, "cpu", torch.float32)
    save_checkpoint(str(tmp_path), cfg, aw0, fw0)

    aw = AttentionWorker.from_pretrained(str(tmp_path), "cpu", torch.float32, max_batch=2,
                                         max_seq=32)
    assert aw.num_layers == cfg.num_hidden_layers and len(aw.layers) == cfg.num_hidden_layers
    torch.testing.assert_close(aw.w.embed, aw0.embed)
    torch.testing.assert_close(aw.w.lm_head, aw0.lm_head)
    assert (aw.cache.max_batch, aw.cache.max_seq) == (2, 32)

    lo, hi = 2, 6
    fw = FFNWorker.from_pretrained(str(tmp_path), "cpu", torch.float32,
                                   expert_range=range(lo, hi))
    assert fw.expert_range == range(lo, hi)
    for l in range(cfg.num_hidden_layers):
        got, want = fw.w.layers[l], fw0.layers[l]
        torch.testing.assert_close(got.post_norm, want.post_norm)
        torch.testing.assert_close(got.w_router, want.w_router)
        torch.testing.assert_close(got.w_gate_up, want.w_gate_up[lo:hi])
        torch.testing.assert_close(got.w_down, want.w_down[lo:hi])

    # a worker built this way runs a layer
    full = FFNWorker.from_pretrained(str(tmp_path), "cpu", torch.float32)
    h = torch.randn(5, cfg.hidden_size, generator=torch.Generator().manual_seed(0))
    out = full.forward_ffn_layer(0, h.clone())
    assert out.shape == h.shape and torch.isfinite(out).all()


def test_workers_from_a_preset():
    cfg = tiny_qwen3_moe()
    aw = AttentionWorker.from_pretrained("tiny", "cpu", torch.float32, max_seq=16)
    fw = FFNWorker.from_pretrained("tiny", "cpu", torch.float32, seed=3)
    assert aw.cfg.hidden_size == cfg.hidden_size and aw.num_layers == cfg.num_hidden_layers
    assert fw.expert_range == range(cfg.num_experts)
    again = FFNWorker.from_pretrained("tiny", "cpu", torch.float32, seed=3)
    assert torch.equal(fw.w.layers[0].w_gate_up, again.w.layers[0].w_gate_up)


def test_reference_per_layer_calls():
    """The reference's worker calls: forward_attention_layer(l, h [B, S, H])
    -> (attn_output, residual), forward_lm_head(h) -> logits [B, S, V],
    get_position_embeddings(h, position_ids), forward_ffn_layer(...,
    return_timing=True) -> (output, FFNStageTiming)."""
    from afd_demo_b200.models.ffn import FFNStageTiming

    cfg = tiny_qwen3_moe()
    aw = AttentionWorker.from_pretrained("tiny", "cpu", torch.float32, max_batch=2, max_seq=16)
    fw = FFNWorker.from_pretrained("tiny", "cpu", torch.float32)
    B, S, H = 2, 5, cfg.hidden_size
    h = torch.randn(B, S, H, generator=torch.Generator().manual_seed(1))

    o, res = aw.forward_attention_layer(0, h)
    o2, res2 = aw.layers[0](h)
    assert o.shape == (B, S, H) and torch.equal(res, h)
    torch.testing.assert_close(o, o2)
    o3, _, cache = aw.forward_attention_layer(0, h, use_cache=True)
    torch.testing.assert_close(o3, o)
    assert cache is aw.cache

    logits = aw.forward_lm_head(h)
    assert logits.shape == (B, S, cfg.vocab_size)
    torch.testing.assert_close(
        logits, aw.lm_head_block([h.reshape(B * S, H)], S, last_only=False).view(B, S, -1))

    pos = torch.arange(S).unsqueeze(0).expand(B, S)
    cos, sin = aw.get_position_embeddings(h, pos)
    assert cos.shape == (B, S, cfg.head_dim)
    cos1, sin1 = aw.get_position_embeddings(pos)
    assert torch.equal(cos, cos1) and torch.equal(sin, sin1)

    x = (h + o).reshape(B * S, H)
    plain = fw.forward_ffn_layer(0, x.clone())
    out, st = fw.forward_ffn_layer(0, x.clone(), return_timing=True)
    assert isinstance(st, FFNStageTiming) and st.router_s >= 0 and st.experts_s >= 0
    torch.testing.assert_close(out, plain)


def test_reference_attribute_names():
    from afd_demo_b200.parallel.micro_batch import MicroBatch, MicroBatchManager

    cfg = tiny_qwen3_moe()
    aw = AttentionWorker.from_pretrained("tiny", "cpu", torch.float32, max_seq=16)
    fw = FFNWorker.from_pretrained("tiny", "cpu", torch.float32)
    for w, layers in ((aw, aw.attention_layers), (fw, fw.ffn_layers)):
        assert w.config is w.cfg and w.hidden_size == cfg.hidden_size
        assert layers is w.layers and w.role_devices == [torch.device("cpu")]
    # the reference's MicroBatch field order (positional construction lines up)
    ids = torch.zeros(2, 3, dtype=torch.long)
    mb = MicroBatch(0, ids, None, None, None)
    assert (mb.position_embeddings, mb.start_time, mb.end_time, mb.batch_offset) == \
        (None, None, None, 0)
    split = MicroBatchManager(2).split_batch(torch.zeros(5, 3, dtype=torch.long))
    assert [m.batch_offset for m in split] == [0, 3]


def test_workers_from_an_hf_model(tmp_path):
    """The reference builds its workers from a loaded HF model. Loaded by
    transformers (experts fused in memory under transformers 5), the workers
    built with ``from_hf_model`` hold the same tensors as those read from the
    checkpoint directory."""
    import transformers

    cfg = tiny_qwen3_moe()
    save_checkpoint(str(tmp_path), cfg, random_attention_weights(cfg, 0, "cpu", torch.float32),
                    random_ffn_weights(cfg, None, 0, "cpu", torch.float32))
    hf = transformers.AutoModelForCausalLM.from_pretrained(str(tmp_path), dtype=torch.float32)

    aw = AttentionWorker.from_hf_model(hf, "cpu", torch.float32, max_seq=16)
    aw_ref = AttentionWorker.from_pretrained(str(tmp_path), "cpu", torch.float32, max_seq=16)
    assert aw.cfg.num_hidden_layers == cfg.num_hidden_layers
    torch.testing.assert_close(aw.w.embed, aw_ref.w.embed, rtol=0, atol=0)
    torch.testing.assert_close(aw.w.layers[1].w_qkv, aw_ref.w.layers[1].w_qkv, rtol=0, atol=0)

    fw = FFNWorker.from_hf_model(hf, "cpu", torch.float32, expert_range=range(1, 3))
    fw_ref = FFNWorker.from_pretrained(str(tmp_path), "cpu", torch.float32,
                                       expert_range=range(1, 3))
    for l in range(cfg.num_hidden_layers):
        for name in ("post_norm", "w_router", "w_gate_up", "w_down"):
            torch.testing.assert_close(getattr(fw.w.layers[l], name),
                                       getattr(fw_ref.w.layers[l], name), rtol=0, atol=0)


def test_state_dict_reader_expert_layouts():
    """Per-expert keys are read as they are; fused transformers-5 expert
    tensors are sliced per expert (gate rows first); other keys are absent."""
    from afd_demo_b200.models.weights import _StateDictReader

    E, I, H = 3, 4, 5
    gu = torch.randn(E, 2 * I, H)
    dn = torch.randn(E, H, I)
    p = "model.layers.0.mlp.experts."
    fused = _StateDictReader({p + "gate_up_proj": gu, p + "down_proj": dn})
    assert torch.equal(fused.get(p + "2.gate_proj.weight"), gu[2, :I])
    assert torch.equal(fused.get(p + "2.up_proj.weight"), gu[2, I:])
    assert torch.equal(fused.get(p + "1.down_proj.weight"), dn[1])
    assert p + "0.gate_proj.weight" in fused and "lm_head.weight" not in fused
    per = _StateDictReader({p + "0.up_proj.weight": gu[0, I:]})
    assert torch.equal(per.get(p + "0.up_proj.weight"), gu[0, I:])
    assert p + "0.gate_proj.weight" not in per


def test_ffn_worker_dense_slices_add_up():
    """Two FFN workers holding the two halves of a dense MLP layer: their
    outputs (residual on the first only) add up to the whole layer's."""
    cfg = tiny_qwen3_moe()
    cfg.mlp_only_layers = [1]
    import tempfile

    d = tempfile.mkdtemp(prefix="afd_dense_")
    save_checkpoint(d, cfg, random_attention_weights(cfg, 0, "cpu", torch.float32),
                    random_ffn_weights(cfg, None, 0, "cpu", torch.float32))
    whole = FFNWorker.from_pretrained(d, "cpu", torch.float32)
    halves = [FFNWorker.from_pretrained(d, "cpu", torch.float32, dense_part=(i, 2))
              for i in range(2)]
    assert halves[0].w.layers[1].w_dense_down.shape[1] == cfg.intermediate_size // 2
    h = torch.randn(4, cfg.hidden_size, generator=torch.Generator().manual_seed(4))
    want = whole.forward_ffn_layer(1, h.clone())
    got = (halves[0].forward_ffn_layer(1, h.clone(), add_residual=True)
           + halves[1].forward_ffn_layer(1, h.clone(), add_residual=False))
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)
