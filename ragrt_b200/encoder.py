"""
Stage 0a: the ColBERT query encoder on the sm_100a kernels of csrc/enc.cu.

Mirrors the reference's fast encoder (src/fast_encoder.py): the same network as a flat
function over fp16 weights -- embeddings + LayerNorm, 12 x [self-attention, LayerNorm, GELU
MLP, LayerNorm], ColBERT's linear 768 -> 128, L2 normalisation -- on fixed [B, 32] token
shapes, captured in one CUDA graph per batch shape.  Every operation runs in
libragrt_b200.so: the seven matrix products per layer on the tensor cores with bias, GELU
and residual fused into their epilogues, the final projection with the fp16 rounding and L2
normalisation fused, LayerNorm and the 32-token attention as their own kernels.

  flat_weights(bert, linear)     the reference's weight dict (fast_encoder.py:31-54)
  flat_forward(W, ids, mask)     [B, L] int64 token ids and attention mask -> [B, L, 128] fp16
  FastQueryEncoder(checkpoint)   encode(text) / encode_batch(texts), as the reference's class
                                 (fast_encoder.py:80-125); `checkpoint` needs .query_tokenizer,
                                 .linear and a BERT model (.bert, .model.bert or .model.LM)

The token ids, [Q] marker and [MASK] padding come from the checkpoint's own tokenizer, as in
the reference; `encode_ids` takes already-tokenized input.
"""
import torch

from . import _lib
from .weft import _need_cuda, _ptr, _stream

EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_GELU_TANH, EPI_BIAS_RESIDUAL, EPI_NORM = 0, 1, 2, 3, 4


def bert_and_linear(checkpoint):
    """(BERT model, ColBERT linear) of a ColBERT checkpoint object (fast_encoder.py:22-28)."""
    bert = getattr(checkpoint, "bert", None)
    if bert is None:
        m = checkpoint.model
        bert = getattr(m, "bert", None) or getattr(m, "LM")
    return bert, checkpoint.linear


def flat_weights(bert, linear, dtype=torch.float16, device="cuda"):
    """fp16 weights of a HuggingFace BertModel state dict + ColBERT's linear, with each layer's
    Q, K and V projections stacked into one [3 D, D] matrix (the reference's layout)."""
    sd = {k: v.detach().to(device=device, dtype=dtype).contiguous() for k, v in bert.state_dict().items()}
    cfg = bert.config
    act = getattr(cfg, "hidden_act", "gelu")
    if act not in ("gelu", "gelu_new", "gelu_python", "gelu_pytorch_tanh"):
        raise RuntimeError(f"unsupported activation {act}")
    W = {"emb_word": sd["embeddings.word_embeddings.weight"],
         "emb_pos": sd["embeddings.position_embeddings.weight"],
         "emb_type": sd["embeddings.token_type_embeddings.weight"][0].contiguous(),
         "emb_ln": (sd["embeddings.LayerNorm.weight"], sd["embeddings.LayerNorm.bias"]),
         "heads": cfg.num_attention_heads, "eps": cfg.layer_norm_eps, "act": act,
         "linear": linear.weight.detach().to(device=device, dtype=dtype).contiguous(), "layers": []}
    for i in range(cfg.num_hidden_layers):
        p = f"encoder.layer.{i}."
        g = lambda n: sd[p + n]
        W["layers"].append({
            "qkv_w": torch.cat([g("attention.self.query.weight"), g("attention.self.key.weight"),
                                g("attention.self.value.weight")], 0).contiguous(),
            "qkv_b": torch.cat([g("attention.self.query.bias"), g("attention.self.key.bias"),
                                g("attention.self.value.bias")], 0).contiguous(),
            "o_w": g("attention.output.dense.weight"), "o_b": g("attention.output.dense.bias"),
            "ln1": (g("attention.output.LayerNorm.weight"), g("attention.output.LayerNorm.bias")),
            "i_w": g("intermediate.dense.weight"), "i_b": g("intermediate.dense.bias"),
            "f_w": g("output.dense.weight"), "f_b": g("output.dense.bias"),
            "ln2": (g("output.LayerNorm.weight"), g("output.LayerNorm.bias")),
        })
    return W


def _gemm(a, w, bias, out, epi, residual=None, ws=None):
    M, K = a.shape
    N = w.shape[0]
    nbytes = ws.numel() * ws.element_size() if ws is not None else 0
    _lib.check(_lib.lib().ragrt_enc_gemm(_ptr(a), _ptr(w), _ptr(bias), _ptr(residual), _ptr(out), M, N, K, epi,
                                         _ptr(ws), nbytes, _stream()))
    return out


def _split_workspace(device):
    """Scratch for the K-split products of small batches.  A product is split only while its
    128 x 128 tiles number at most half the SMs, into at most SMs / tiles slices, so the fp32
    partials never exceed SMs x 128 x 128 values (9.7 MB on 148 SMs)."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return torch.empty(sms * 128 * 128, dtype=torch.float32, device=device)


def _gemm_residual_ln(a, w, bias, residual, ln, eps, tmp, out, ws=None):
    M, K = a.shape
    N = w.shape[0]
    nbytes = ws.numel() * ws.element_size() if ws is not None else 0
    _lib.check(_lib.lib().ragrt_enc_gemm_residual_ln(_ptr(a), _ptr(w), _ptr(bias), _ptr(residual), _ptr(ln[0]),
                                                     _ptr(ln[1]), float(eps), _ptr(tmp), _ptr(out), M, N, K,
                                                     _ptr(ws), nbytes, _stream()))
    return out


def _layernorm(x, ln, eps, out):
    _lib.check(_lib.lib().ragrt_enc_layernorm(_ptr(x), _ptr(ln[0]), _ptr(ln[1]), float(eps), _ptr(out), x.shape[0],
                                              x.shape[1], _stream()))
    return out


def flat_forward(W, ids, mask):
    """ids, mask [B, L] (int64, on the weights' device) -> unit ColBERT query vectors
    [B, L, dim] fp16.  Needs L = 32, hidden size 768 and head size 64 (BERT-base)."""
    _need_cuda(ids, mask, W["emb_word"])
    ids = ids.to(torch.int64).contiguous()
    mask = mask.to(torch.int64).contiguous()
    B, L = ids.shape
    if mask.shape != ids.shape or L > W["emb_pos"].shape[0]:
        raise RuntimeError(f"ids / mask must be [B, L] with L <= {W['emb_pos'].shape[0]} positions")
    M = B * L
    D = W["emb_word"].shape[1]
    H = W["heads"]
    eps = W["eps"]
    dev = ids.device
    x = torch.empty(M, D, dtype=torch.float16, device=dev)
    y = torch.empty(M, D, dtype=torch.float16, device=dev)
    ctx = torch.empty(M, D, dtype=torch.float16, device=dev)
    qkv = torch.empty(M, 3 * D, dtype=torch.float16, device=dev)
    h = torch.empty(M, W["layers"][0]["i_w"].shape[0], dtype=torch.float16, device=dev)
    ws = _split_workspace(dev)
    _lib.check(_lib.lib().ragrt_enc_embed(_ptr(ids), _ptr(W["emb_word"]), _ptr(W["emb_pos"]), _ptr(W["emb_type"]),
                                          _ptr(W["emb_ln"][0]), _ptr(W["emb_ln"][1]), float(eps),
                                          W["emb_word"].shape[0], B, L, D, _ptr(x), _stream()))
    gelu = EPI_BIAS_GELU_TANH if W["act"] in ("gelu_new", "gelu_pytorch_tanh") else EPI_BIAS_GELU
    for lw in W["layers"]:
        _gemm(x, lw["qkv_w"], lw["qkv_b"], qkv, EPI_BIAS, ws=ws)
        _lib.check(_lib.lib().ragrt_enc_attention(_ptr(qkv), _ptr(mask), _ptr(ctx), B, L, H, D, _stream()))
        _gemm_residual_ln(ctx, lw["o_w"], lw["o_b"], x, lw["ln1"], eps, y, x, ws=ws)
        _gemm(x, lw["i_w"], lw["i_b"], h, gelu, ws=ws)
        _gemm_residual_ln(h, lw["f_w"], lw["f_b"], x, lw["ln2"], eps, y, x, ws=ws)
    out = torch.empty(M, W["linear"].shape[0], dtype=torch.float16, device=dev)
    _gemm(x, W["linear"], None, out, EPI_NORM, ws=ws)
    return out.view(B, L, -1)


class FastQueryEncoder:
    """encode(text) -> ([32, 128] fp16, ntok); encode_batch(texts) -> ([B, 32, 128] fp16, ntoks)."""

    def __init__(self, checkpoint=None, device="cuda", use_graphs=True, weights=None, tokenizer=None):
        self.tok = tokenizer if tokenizer is not None else getattr(checkpoint, "query_tokenizer", None)
        if weights is None:
            bert, linear = bert_and_linear(checkpoint)
            weights = flat_weights(bert, linear, device=device)
        self.W = weights
        self.device, self.use_graphs = device, use_graphs
        self.graphs = {}

    def tokenize(self, texts):
        if self.tok is None:
            raise RuntimeError("no query tokenizer: pass token ids to encode_ids")
        return self.tok.tensorize(list(texts))

    def _graph(self, B, L):
        key = (B, L)
        if key not in self.graphs:
            ids = torch.zeros(B, L, dtype=torch.int64, device=self.device)
            mask = torch.ones(B, L, dtype=torch.int64, device=self.device)
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s), torch.no_grad():
                for _ in range(2):
                    flat_forward(self.W, ids, mask)
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g), torch.no_grad():
                out = flat_forward(self.W, ids, mask)
            self.graphs[key] = (g, ids, mask, out)
        return self.graphs[key]

    @torch.no_grad()
    def encode_ids(self, ids, mask):
        """Token ids and attention mask [B, L] (host or device) -> [B, L, 128] fp16 on the device."""
        if not self.use_graphs:
            return flat_forward(self.W, ids.to(self.device), mask.to(self.device))
        g, gi, gm, out = self._graph(*ids.shape)
        gi.copy_(ids, non_blocking=True)
        gm.copy_(mask, non_blocking=True)
        g.replay()
        return out.clone()

    @torch.no_grad()
    def encode_batch(self, texts):
        ids, mask = self.tokenize(texts)
        ntoks = mask.sum(1).tolist()
        return self.encode_ids(ids, mask), ntoks

    def encode(self, text):
        Q, ntoks = self.encode_batch([text])
        return Q[0].contiguous(), int(ntoks[0])
