"""The maximum corpus size of the posting format, on the CPU: 2^24 passages with pids up to
2^24 - 1 (ragrt_index_lib.py:23-24, 167-185).  The index builder packs the top pids into
their three little-endian bytes, and the oracle over the full pid space gives what it gives
over the same documents packed densely, with pids mapped (the map is monotonic, so the
ranking rules keep the same order)."""
import numpy as np

from oracle import oracle as O
from tests.helpers import MAX_PASSAGES, max_pid_corpus, oracle_index, small_corpus

NC, K, K_TOP = 16, 300, 10


def _unpack(p24):
    b = p24.numpy().astype(np.int64).reshape(-1, 3)
    return b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)


def test_top_pids_pack_into_24_bits():
    d, _, _, pid_map = max_pid_corpus()
    pids = _unpack(d["csr_packed_24"])
    assert pids.max() == MAX_PASSAGES - 1
    assert set(np.unique(pids).tolist()) == set(pid_map.numpy().tolist())   # every doc has tokens


def test_oracle_over_full_pid_space_equals_dense_corpus():
    d, Q, E, pid_map = max_pid_corpus()
    d0, Q0, E0, _ = small_corpus(num_docs=2000, nq=4)
    assert E == E0
    big, small = oracle_index(d), oracle_index(d0)
    pm = pid_map.numpy()
    q = Q.numpy()
    ntok = np.array([32, 29, 32, 23], np.int32)
    masks = np.array([0, 1, 0, 2], np.uint32)
    ids, sc, _ = O.weft_search(big, q, ntok, NC, E, masks, K, K_TOP)
    ids0, sc0, _ = O.weft_search(small, q, ntok, NC, E, masks, K, K_TOP)
    mapped = np.where(ids0 >= 0, pm[np.maximum(ids0, 0)], -1)
    assert np.array_equal(ids, mapped)
    assert np.array_equal(sc, sc0)
