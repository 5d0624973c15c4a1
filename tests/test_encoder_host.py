"""Host side of Stage 0a, no GPU: the weight layout flat_weights builds from a HuggingFace
BertModel (the reference's layout, fast_encoder.py:31-54: Q, K, V stacked in that order, each
layer's dense and LayerNorm tensors by name) and the drop-in module's surface."""
import inspect

import pytest
import torch

from ragrt_b200 import encoder


@pytest.fixture(scope="module")
def small_bert():
    transformers = pytest.importorskip("transformers")
    cfg = transformers.BertConfig(hidden_size=128, num_hidden_layers=2, num_attention_heads=2,
                                  intermediate_size=256, vocab_size=500, max_position_embeddings=64)
    torch.manual_seed(0)
    return transformers.BertModel(cfg, add_pooling_layer=False).eval(), torch.nn.Linear(128, 32, bias=False)


def test_flat_weights_layout(small_bert):
    bert, linear = small_bert
    W = encoder.flat_weights(bert, linear, device="cpu")
    sd = {k: v.half() for k, v in bert.state_dict().items()}
    assert W["heads"] == 2 and W["eps"] == bert.config.layer_norm_eps and W["act"] == "gelu"
    assert torch.equal(W["emb_word"], sd["embeddings.word_embeddings.weight"])
    assert torch.equal(W["emb_type"], sd["embeddings.token_type_embeddings.weight"][0])
    assert torch.equal(W["linear"], linear.weight.half())
    assert len(W["layers"]) == 2
    for i, lw in enumerate(W["layers"]):
        p = f"encoder.layer.{i}."
        q, k, v = lw["qkv_w"].split(128, 0)
        assert torch.equal(q, sd[p + "attention.self.query.weight"])
        assert torch.equal(k, sd[p + "attention.self.key.weight"])
        assert torch.equal(v, sd[p + "attention.self.value.weight"])
        assert torch.equal(lw["qkv_b"][256:], sd[p + "attention.self.value.bias"])
        assert torch.equal(lw["i_w"], sd[p + "intermediate.dense.weight"])
        assert torch.equal(lw["f_w"], sd[p + "output.dense.weight"])
        assert torch.equal(lw["ln2"][0], sd[p + "output.LayerNorm.weight"])
        for t in (lw["qkv_w"], lw["o_w"], lw["i_w"], lw["f_w"]):
            assert t.is_contiguous() and t.dtype == torch.float16


def test_flat_forward_refuses_host_tensors(small_bert):
    bert, linear = small_bert
    W = encoder.flat_weights(bert, linear, device="cpu")
    ids = torch.zeros(1, 32, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="CUDA"):
        encoder.flat_forward(W, ids, torch.ones_like(ids))


def test_fast_encoder_dropin_surface():
    import importlib.util
    import os
    path = os.path.join(os.path.dirname(encoder.__file__), "compat", "fast_encoder.py")
    spec = importlib.util.spec_from_file_location("fast_encoder", path)
    fe = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fe)
    for name in ("bert_and_linear", "flat_weights", "flat_forward", "FastQueryEncoder"):
        assert hasattr(fe, name)
    assert list(inspect.signature(fe.flat_forward).parameters) == ["W", "ids", "mask"]
    assert list(inspect.signature(fe.FastQueryEncoder.__init__).parameters)[:4] == \
        ["self", "checkpoint", "device", "use_graphs"]
    for m in ("tokenize", "encode_batch", "encode", "encode_ids"):
        assert callable(getattr(fe.FastQueryEncoder, m))


def test_tokenizer_required_for_text():
    enc = encoder.FastQueryEncoder(weights={"layers": []}, device="cpu")
    with pytest.raises(RuntimeError, match="tokenizer"):
        enc.encode_batch(["what is colbert"])
