"""Independent oracle: HF transformers' own Qwen3-MoE, the model code the
reference's workers call (src/model/attention_worker.py:127,
src/model/ffn_worker.py:98-107), loads a checkpoint that this framework's writer
produced in the Qwen3-MoE safetensors layout (per-expert
`mlp.experts.{e}.{gate,up,down}_proj.weight`, sharded index). Its logits and
greedy tokens must match this framework's CPU path in every schedule."""

import pytest
import torch

transformers = pytest.importorskip("transformers")

from afd_demo_b200.config import tiny_qwen3_moe  # noqa: E402
from afd_demo_b200.models import DisaggregatedQwenModel  # noqa: E402
from afd_demo_b200.models.weights import write_random_checkpoint  # noqa: E402


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("ckpt"))
    cfg = tiny_qwen3_moe()
    write_random_checkpoint(path, cfg, seed=0, dtype=torch.float32)
    hf = transformers.AutoModelForCausalLM.from_pretrained(path, dtype=torch.float32)
    hf.eval()
    ours = DisaggregatedQwenModel.from_pretrained(path, device="cpu", dtype=torch.float32,
                                                  max_seq_len=64, max_batch_size=4)
    ids = torch.randint(0, cfg.vocab_size, (4, 16), generator=torch.Generator().manual_seed(0))
    return hf, ours, ids


def test_hf_reads_the_checkpoint_layout(models):
    hf, ours, _ = models
    assert type(hf).__name__ == "Qwen3MoeForCausalLM"
    assert hf.config.num_experts == ours.config.num_experts
    assert hf.config.norm_topk_prob is True


@pytest.mark.parametrize("mode,nmb", [("serial", 1), ("dbo", 2)])
def test_last_position_logits_match_hf(models, mode, nmb):
    hf, ours, ids = models
    with torch.no_grad():
        ref = hf(ids).logits[:, -1].float()
    out = ours.run_forward(ids, mode, nmb, reset_cache=True).float()
    assert out.shape == ref.shape
    assert (out - ref).abs().max().item() < 1e-3 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("dbo,crosslayer", [(False, False), (True, False), (True, True)])
def test_greedy_tokens_match_hf(models, dbo, crosslayer):
    hf, ours, ids = models
    with torch.no_grad():
        ref = hf.generate(ids, max_new_tokens=8, do_sample=False, pad_token_id=0,
                          eos_token_id=None)
    out = ours.generate(ids, max_new_tokens=8, do_sample=False, use_decode_dbo=dbo,
                        decode_use_crosslayer=crosslayer)
    assert torch.equal(out[:, ids.shape[1]:].cpu(), ref[:, ids.shape[1]:])


def test_reads_a_checkpoint_saved_by_transformers(models, tmp_path):
    """The other direction: transformers 5 saves a single `model.safetensors`
    and names the expert count `num_local_experts`; the loader reads both."""
    hf, _, ids = models
    hf.save_pretrained(str(tmp_path))
    again = DisaggregatedQwenModel.from_pretrained(str(tmp_path), device="cpu",
                                                   dtype=torch.float32, max_seq_len=64,
                                                   max_batch_size=4)
    assert again.config.num_experts == hf.config.num_experts
    with torch.no_grad():
        ref = hf(ids).logits[:, -1].float()
    out = again.run_forward(ids, "serial", 1, reset_cache=True).float()
    assert (out - ref).abs().max().item() < 1e-3 * max(1.0, ref.abs().max().item())


def test_dense_mlp_layers_match_hf(tmp_path):
    """`mlp_only_layers` layers are a dense SwiGLU MLP (HF `Qwen3MoeMLP`)."""
    cfg = tiny_qwen3_moe()
    cfg.mlp_only_layers = [1]
    write_random_checkpoint(str(tmp_path), cfg, seed=1, dtype=torch.float32)
    hf = transformers.AutoModelForCausalLM.from_pretrained(str(tmp_path), dtype=torch.float32)
    assert type(hf.model.layers[1].mlp).__name__ == "Qwen3MoeMLP"
    ours = DisaggregatedQwenModel.from_pretrained(str(tmp_path), device="cpu",
                                                  dtype=torch.float32, max_seq_len=64,
                                                  max_batch_size=2)
    ids = torch.randint(0, cfg.vocab_size, (2, 16), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        ref = hf(ids).logits[:, -1].float()
    out = ours.run_forward(ids, "dbo", 2, reset_cache=True).float()
    assert (out - ref).abs().max().item() < 1e-3 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("tied", [False, True])
def test_dense_qwen3_checkpoint_matches_hf(tmp_path, tied):
    """A dense Qwen3 model (``Qwen3ForCausalLM``: no router, no expert count
    in its config), saved by transformers, loads as a model whose every FFN
    layer is a dense MLP; logits and greedy tokens match HF's own. With tied
    embeddings the checkpoint has no ``lm_head.weight`` and the embedding is
    the LM head."""
    hcfg = transformers.Qwen3Config(vocab_size=512, hidden_size=128, intermediate_size=256,
                                    num_hidden_layers=2, num_attention_heads=4,
                                    num_key_value_heads=2, head_dim=32,
                                    max_position_embeddings=256, tie_word_embeddings=tied)
    torch.manual_seed(0)
    hf = transformers.Qwen3ForCausalLM(hcfg).float().eval()
    hf.save_pretrained(str(tmp_path))
    ours = DisaggregatedQwenModel.from_pretrained(str(tmp_path), device="cpu",
                                                  dtype=torch.float32, max_seq_len=64,
                                                  max_batch_size=2)
    assert ours.config.num_experts == 0 and ours.config.model_type == "qwen3"
    assert ours.ffn_worker.w.layers[0].w_router is None
    ids = torch.randint(0, 512, (2, 12), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        ref = hf(ids).logits[:, -1].float()
        want = hf.generate(ids, max_new_tokens=6, do_sample=False)
    for mode, nmb in (("serial", 1), ("dbo", 2)):
        out = ours.run_forward(ids, mode, nmb, reset_cache=True).float()
        assert (out - ref).abs().max().item() < 1e-3 * max(1.0, ref.abs().max().item())
    got = ours.generate(ids, max_new_tokens=6, do_sample=False, use_decode_dbo=False)
    assert torch.equal(got, want)


@pytest.mark.parametrize("side", ["right", "left"])
def test_padding_mask_matches_hf(models, side):
    """Prefill with a padding mask (the reference's `--prefill-seq-len`
    max_length padding): padded keys are hidden, positions stay 0..S-1, as
    HF computes for `model(ids, attention_mask=mask)`."""
    hf, ours, ids = models
    B, S = ids.shape
    lens = torch.tensor([S, S - 3, S - 7, 5])
    mask = torch.zeros(B, S, dtype=torch.long)
    for b in range(B):
        if side == "right":
            mask[b, :lens[b]] = 1
        else:
            mask[b, S - lens[b]:] = 1
    with torch.no_grad():
        ref = hf(ids, attention_mask=mask).logits.float()
    full = ours.forward(ids, attention_mask=mask).float()
    for b in range(B):
        # rows whose query sees at least one key (left padding: the real tokens)
        rows = slice(0, S) if side == "right" else slice(S - int(lens[b]), S)
        d = (full[b, rows] - ref[b, rows]).abs().max().item()
        assert d < 1e-3 * max(1.0, ref[b, rows].abs().max().item()), (b, d)
    for mode, nmb in (("serial", 1), ("dbo", 2)):
        last = ours.run_forward(ids, mode, nmb, reset_cache=True, attention_mask=mask).float()
        assert (last - ref[:, -1]).abs().max().item() < 1e-3 * max(1.0, ref[:, -1].abs().max().item())


def test_forward_prefill_and_decode_shapes_match_hf(models):
    """forward_prefill returns logits for every position and forward_decode
    [B, 1, V], the reference's shapes; both equal HF's logits."""
    hf, ours, ids = models
    with torch.no_grad():
        ref = hf(ids).logits.float()
    full = ours.forward_prefill(ids).float()
    assert full.shape == ref.shape
    assert (full - ref).abs().max().item() < 1e-3 * max(1.0, ref.abs().max().item())
    nxt = ref[:, -1].argmax(-1, keepdim=True)
    step = ours.forward_decode(nxt).float()
    with torch.no_grad():
        ref2 = hf(torch.cat([ids, nxt], 1)).logits[:, -1:].float()
    assert step.shape == ref2.shape
    assert (step - ref2).abs().max().item() < 1e-3 * max(1.0, ref2.abs().max().item())


def _head(model, h):
    aw = model.attention_worker
    B, S, H = h.shape
    return aw.lm_head_block([h.reshape(B * S, H)], S, last_only=False).view(B, S, -1)


def test_per_layer_entry_points_match_hf(models):
    """forward_layer_sync (whole sequence, no cache) and
    forward_layer_with_cache (prefill, then a decode token), layer by layer
    from the embedding to the LM head, as the reference's per-layer path."""
    hf, ours, ids = models
    B, S = ids.shape
    emb = lambda t: ours.attention_worker.embed(t).view(t.shape[0], t.shape[1], -1)  # noqa: E731
    with torch.no_grad():
        ref = hf(ids).logits.float()
    h = emb(ids)
    for l in range(ours.num_layers):
        h = ours.forward_layer_sync(l, h)
    got = _head(ours, h).float()
    assert (got - ref).abs().max().item() < 1e-3 * max(1.0, ref.abs().max().item())
    ours.reset_kv_cache()
    h = emb(ids)
    for l in range(ours.num_layers):
        h = ours.forward_layer_with_cache(l, h)
    assert ours.kv_cache.get_seq_length() == S
    nxt = ref[:, -1].argmax(-1, keepdim=True)
    h = emb(nxt)
    for l in range(ours.num_layers):
        h = ours.forward_layer_with_cache(l, h)
    step = _head(ours, h).float()
    with torch.no_grad():
        ref2 = hf(torch.cat([ids, nxt], 1)).logits[:, -1:].float()
    assert (step - ref2).abs().max().item() < 1e-3 * max(1.0, ref2.abs().max().item())


def test_layer_views_match_hf_and_fused_path(models):
    """AttentionLayer / FFNLayer (the reference's per-layer modules): the
    FFN layer equals HF's post-attention norm + MoE block + residual; the
    attention layer's (attn_output + residual) equals the fused layer
    output."""
    hf, ours, ids = models
    B, S = ids.shape
    aw, fw = ours.attention_worker, ours.ffn_worker
    x = aw.embed(ids).view(B, S, -1)
    blk = hf.model.layers[0]
    with torch.no_grad():
        ref_ffn = x + blk.mlp(blk.post_attention_layernorm(x))
    got, st = fw.layers[0](x, return_timing=True)
    assert (got - ref_ffn).abs().max().item() < 1e-3 * max(1.0, ref_ffn.abs().max().item())
    assert fw.layers[0].is_sparse_moe and st.router_s >= 0.0 and st.experts_s > 0.0
    ours.reset_kv_cache()
    attn, res = aw.layers[0](x)
    ours.reset_kv_cache()
    h = aw.attention_block(0, [x.reshape(B * S, -1)], 0, S, start_pos=0)
    torch.testing.assert_close((attn + res).reshape(B * S, -1), h, rtol=1e-5, atol=1e-5)
    ours.reset_kv_cache()
    attn2, res2, cache = aw.layers[0](x, use_cache=True)
    assert cache is aw.cache and torch.equal(attn2, attn) and torch.equal(res2, res)
