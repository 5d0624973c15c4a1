"""No CPU fallback, no silent misconfiguration (no GPU needed): a missing library raises,
CPU tensors are refused by every op, and the drop-in rejects what the reference rejects before
any device work."""
import os
import sys

import pytest
import torch

from ragrt_b200 import _lib, weft

COMPAT = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "ragrt_b200", "compat")


def test_missing_library_raises(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "libragrt_b200.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


def test_ops_refuse_host_tensors():
    Q = torch.zeros(1, 32, 128, dtype=torch.float16)
    C = torch.zeros(64, 128, dtype=torch.float16)
    pids = torch.zeros(1, 4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        weft.centroid_topk(Q, C, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        weft.final_topk(pids, torch.zeros(1, 4), 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        weft.tile_maxsim_exact(Q, pids, torch.zeros(2, dtype=torch.int64), torch.ones(1, dtype=torch.int32),
                               torch.zeros(1, 128, dtype=torch.float16))


def test_dropin_rejects_bad_configuration():
    if COMPAT not in sys.path:
        sys.path.insert(0, COMPAT)
    import rtrag_corr_3d as R
    idx = R.CorrIndex3D("ignored.ptx")
    with pytest.raises(RuntimeError):
        idx.build(torch.zeros(16, 8, 3))                    # codebooks must be [32, E, 3]
    with pytest.raises(RuntimeError):
        idx.set_stage1_mode(3)
    with pytest.raises(RuntimeError):
        idx.set_geometry(5)
    with pytest.raises(NotImplementedError):
        idx.set_residual_lut(torch.zeros(4))               # residual scoring is another engine
    with pytest.raises(RuntimeError, match="bound"):
        idx.search_single_query_native(None, None, torch.zeros(4, 32, 3), None, None, 8, 10, 5)
    idx.build(torch.zeros(32, 8, 3))
    assert idx.info()["num_entries"] == 8


class _Stop(Exception):
    pass


def test_every_tensor_argument_is_device_checked(monkeypatch):
    """Each entry point hands ALL of its tensor arguments -- optional ones such as ntok, masks,
    predicates and output buffers included -- to the device check before any pointer reaches
    the library: a host tensor there would be dereferenced on the device."""
    seen = []

    def record(*ts):
        seen.append(ts)
        raise _Stop

    monkeypatch.setattr(weft, "_need_cuda", record)
    T = [torch.zeros(1) for _ in range(16)]

    def checked(fn, *args, expect, **kw):
        seen.clear()
        with pytest.raises(_Stop):
            fn(*args, **kw)
        got = {id(t) for t in seen[0] if t is not None}
        missing = [i for i, t in enumerate(expect) if id(t) not in got]
        assert not missing, (fn.__name__, missing)

    checked(weft.centroid_topk, T[0], T[1], 8, ntok=T[2], expect=T[:3])
    checked(weft.tile_maxsim, *T[:10], expect=T[:10])
    checked(weft.tile_maxsim_exact, *T[:5], expect=T[:5])
    checked(weft.final_topk, T[0], T[1], 4, preds=T[2], masks=T[3], expect=T[:4])
    checked(weft.WeftIndex, *T[:13], doc_predicates=T[13], expect=T[:14])
    ix = object.__new__(weft.WeftIndex)
    checked(ix.candidates, T[0], T[1], 10, ntok=T[2], masks=T[3], expect=T[:4])
    checked(ix.search, T[0], ntok=T[1], masks=T[2], out=(T[3], T[4]), expect=T[:5])
    checked(ix.search_profiled, T[0], [], ntok=T[1], masks=T[2], out=(T[3], T[4]), expect=T[:5])


def test_device_check_refuses_host_tensors_among_cuda_ones():
    with pytest.raises(RuntimeError, match="CUDA"):
        weft._need_cuda(None, torch.zeros(1))
    weft._need_cuda(None, None)                                  # nothing to check
