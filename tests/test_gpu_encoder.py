"""Stage 0a (the ColBERT query encoder) on the sm_100a kernels.

References: the tensor-core GEMM and its epilogues against fp32 torch on the same fp16
inputs; the whole encoder against HuggingFace's BertModel in fp32 (a randomly initialised
BERT-base with the same fp16-rounded weights; there is no network for a checkpoint) followed
by ColBERT's linear and L2 normalisation -- the check the reference's own encoder test makes
(its flat forward against BertModel).  Tolerances: fp16 storage of the activations between
the 12 layers; each output token must keep a cosine similarity of at least 0.999 with the
fp32 reference.
"""
import pytest
import torch
import torch.nn.functional as F

from ragrt_b200 import _lib, encoder

pytestmark = pytest.mark.gpu


def _gemm(a, w, bias=None, residual=None, epi=encoder.EPI_BIAS):
    out = torch.empty(a.shape[0], w.shape[0], dtype=torch.float16, device="cuda")
    return encoder._gemm(a, w, bias, out, epi, residual=residual)


@pytest.mark.parametrize("M", [32, 96, 200, 1024])
@pytest.mark.parametrize("epi", [encoder.EPI_BIAS, encoder.EPI_BIAS_GELU, encoder.EPI_BIAS_GELU_TANH,
                                 encoder.EPI_BIAS_RESIDUAL])
def test_gemm_epilogues(M, epi):
    g = torch.Generator(device="cuda").manual_seed(M + 7 * epi)
    N, K = 256, 768
    a = torch.randn(M, K, generator=g, device="cuda").half()
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.05).half()
    b = (torch.randn(N, generator=g, device="cuda") * 0.1).half()
    r = torch.randn(M, N, generator=g, device="cuda").half()
    got = _gemm(a, w, b, r if epi == encoder.EPI_BIAS_RESIDUAL else None, epi).float()
    ref = a.float() @ w.float().t() + b.float()
    if epi == encoder.EPI_BIAS_GELU:
        ref = F.gelu(ref)
    elif epi == encoder.EPI_BIAS_GELU_TANH:
        ref = F.gelu(ref, approximate="tanh")
    elif epi == encoder.EPI_BIAS_RESIDUAL:
        ref = ref + r.float()
    err = (got - ref).abs()
    assert err.max().item() <= 2e-3 * ref.abs().max().item() + 2e-3, err.max().item()


@pytest.mark.parametrize("M,N,K", [(32, 768, 3072), (32, 3072, 768), (200, 768, 768), (64, 128, 768)])
@pytest.mark.parametrize("epi", [encoder.EPI_BIAS_GELU, encoder.EPI_BIAS_RESIDUAL, encoder.EPI_NORM])
def test_gemm_split_k_equals_reference(M, N, K, epi):
    """Small M: the product is split along K over more CTAs and summed in fp32 by a second
    kernel that applies the epilogue."""
    if epi == encoder.EPI_NORM and N != 128:
        pytest.skip("the normalising epilogue is for the 128-wide projection")
    g = torch.Generator(device="cuda").manual_seed(M * 3 + N + epi)
    a = torch.randn(M, K, generator=g, device="cuda").half()
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.05).half()
    b = None if epi == encoder.EPI_NORM else (torch.randn(N, generator=g, device="cuda") * 0.1).half()
    r = torch.randn(M, N, generator=g, device="cuda").half()
    ws = encoder._split_workspace(torch.device("cuda"))
    out = torch.empty(M, N, dtype=torch.float16, device="cuda")
    got = encoder._gemm(a, w, b, out, epi, residual=r if epi == encoder.EPI_BIAS_RESIDUAL else None, ws=ws).float()
    ref = a.float() @ w.float().t()
    if epi == encoder.EPI_NORM:
        ref = F.normalize(ref.half().float(), dim=-1)
    else:
        ref = ref + b.float()
        ref = F.gelu(ref) if epi == encoder.EPI_BIAS_GELU else ref + r.float()
    err = (got - ref).abs().max().item()
    assert err <= 2e-3 * ref.abs().max().item() + 2e-3, err


@pytest.mark.parametrize("M,K", [(64, 768), (32, 3072), (4096, 768)])
def test_gemm_residual_layernorm(M, K):
    """LN(A W^T + b + residual) written over the residual: split K with the LayerNorm fused into
    the reduction (small M), or the residual epilogue then the LayerNorm kernel (large M)."""
    g = torch.Generator(device="cuda").manual_seed(M + K)
    N = 768
    a = torch.randn(M, K, generator=g, device="cuda").half()
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.03).half()
    b = (torch.randn(N, generator=g, device="cuda") * 0.1).half()
    x = torch.randn(M, N, generator=g, device="cuda").half()
    gamma = (1 + 0.1 * torch.randn(N, generator=g, device="cuda")).half()
    beta = (0.1 * torch.randn(N, generator=g, device="cuda")).half()
    ref = F.layer_norm((a.float() @ w.float().t() + b.float() + x.float()).half().float(), (N,), gamma.float(),
                       beta.float(), eps=1e-12)
    tmp = torch.empty_like(x)
    ws = encoder._split_workspace(torch.device("cuda"))
    got = encoder._gemm_residual_ln(a, w, b, x, (gamma, beta), 1e-12, tmp, x, ws=ws).float()
    assert (got - ref).abs().max().item() < 2e-2


def test_gemm_norm_epilogue():
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(160, 768, generator=g, device="cuda").half()
    w = (torch.randn(128, 768, generator=g, device="cuda") * 0.05).half()
    got = _gemm(a, w, None, None, encoder.EPI_NORM).float()
    ref = F.normalize((a.float() @ w.float().t()).half().float(), dim=-1)
    assert (got - ref).abs().max().item() < 2e-3
    assert torch.allclose(got.norm(dim=-1), torch.ones(160, device="cuda"), atol=2e-3)


def test_gemm_rejects_bad_shapes():
    a = torch.zeros(64, 100, dtype=torch.float16, device="cuda")
    w = torch.zeros(128, 100, dtype=torch.float16, device="cuda")
    with pytest.raises(_lib.RagrtError):
        _gemm(a, w)


@pytest.fixture(scope="module")
def bert():
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(0)
    cfg = transformers.BertConfig()                     # BERT-base: 12 layers, 768 hidden, 12 heads
    model = transformers.BertModel(cfg, add_pooling_layer=False).eval()
    with torch.no_grad():                               # non-trivial LayerNorms and biases
        for name, p in model.named_parameters():
            if "LayerNorm.weight" in name:
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
            elif name.endswith("bias"):
                p.copy_(0.02 * torch.randn_like(p))
        for p in model.parameters():                    # the values the fp16 kernels see
            p.copy_(p.half().float())
    linear = torch.nn.Linear(768, 128, bias=False)
    with torch.no_grad():
        linear.weight.copy_((0.05 * torch.randn(128, 768)).half().float())
    return model.cuda(), linear.cuda()


def _inputs(B, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(1000, 30000, (B, 32), generator=g)
    ids[:, 0], ids[:, 1] = 101, 1                       # [CLS] and the query marker
    mask = torch.ones(B, 32, dtype=torch.int64)
    for b in range(B):                                  # ColBERT pads with [MASK] tokens it does not attend to
        n = int(torch.randint(3, 33, (1,), generator=g))
        ids[b, n:] = 103
        mask[b, n:] = 0
    return ids.cuda(), mask.cuda()


def _reference(model, linear, ids, mask):
    with torch.no_grad():
        h = model(input_ids=ids, attention_mask=mask).last_hidden_state
        return F.normalize(linear(h), dim=-1)


def test_encoder_matches_bert_fp32(bert):
    model, linear = bert
    W = encoder.flat_weights(model, linear)
    ids, mask = _inputs(16, 1)
    got = encoder.flat_forward(W, ids, mask).float()
    ref = _reference(model, linear, ids, mask)
    cos = (got * ref).sum(-1) / got.norm(dim=-1)
    assert cos.min().item() >= 0.999, cos.min().item()
    assert (got - ref).abs().max().item() < 0.05


def test_encoder_graph_replay_equals_eager(bert):
    model, linear = bert
    enc = encoder.FastQueryEncoder(weights=encoder.flat_weights(model, linear), use_graphs=True)
    for seed in (2, 3):                                 # the second replay sees new inputs
        ids, mask = _inputs(8, seed)
        got = enc.encode_ids(ids.cpu(), mask.cpu())
        ref = encoder.flat_forward(enc.W, ids, mask)
        assert torch.equal(got, ref)


def test_encoder_bad_token_id_raises_device_flag(bert):
    model, linear = bert
    W = encoder.flat_weights(model, linear)
    ids, mask = _inputs(2, 4)
    ids[1, 5] = 10 ** 6
    _lib.lib().ragrt_device_error(1)
    encoder.flat_forward(W, ids, mask)
    torch.cuda.synchronize()
    assert _lib.lib().ragrt_device_error(1) == 4
