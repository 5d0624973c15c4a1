"""Drop-in for the reference's `fast_encoder` module (src/fast_encoder.py): the ColBERT query
encoder with the same names and signatures -- bert_and_linear(checkpoint), flat_weights(bert,
linear, dtype, device), flat_forward(W, ids, mask) and FastQueryEncoder(checkpoint, device,
use_graphs) with tokenize / encode_batch / encode -- running on this build's sm_100a kernels
(ragrt_b200.encoder).  FastQueryEncoder also takes `weights=` / `tokenizer=` and offers
encode_ids(ids, mask) for already-tokenized input."""
from ragrt_b200.encoder import FastQueryEncoder, bert_and_linear, flat_forward, flat_weights  # noqa: F401
