"""Host-side eligibility rules of the symmetric TP workspace (no GPU: a stand-in tensor object).

The row-statistic exchanges store partials for every row of whole 64-row blocks, so their
capacity checks must count rows rounded up to 64: q and k of one call occupy two block-aligned
slab ranges, and the cross-entropy exchange stores three floats per (padded) row."""

import torch

from cq_pretrain_b200.parallel import symmetric


class _Rows:
    """Just enough of a CUDA bf16 [rows, width] tensor for the eligibility checks."""

    def __init__(self, rows, width, stride=None, ptr=4096):
        self.shape = (rows, width)
        self._stride = (stride or width, 1)
        self._ptr = ptr
        self.is_cuda = True
        self.dtype = torch.bfloat16

    def dim(self):
        return 2

    def stride(self, i=None):
        return self._stride if i is None else self._stride[i]

    def data_ptr(self):
        return self._ptr


def _workspace(stat_rows):
    ws = object.__new__(symmetric.SymmetricWorkspace)   # eligibility only: no peer memory
    ws.stat_rows = stat_rows
    return ws


def test_statistics_capacity_counts_whole_blocks(monkeypatch):
    monkeypatch.setattr(symmetric._ext, "has", lambda name: True)
    ws = _workspace(stat_rows=4096)
    assert ws.supports_rms(_Rows(4096, 768))
    assert ws.supports_qk(_Rows(2048, 768), _Rows(2048, 768, stride=1536))
    # 2,040 rows pad to 2,048 per tensor: two of them still fit; 2,049 rows pad to 2,112 and do not
    assert ws.supports_qk(_Rows(2040, 768), _Rows(2040, 768))
    assert not ws.supports_qk(_Rows(2049, 768), _Rows(2049, 768))
    # cross-entropy: three floats per padded row
    assert ws.supports_ce(1344)            # 1,344 rows = 21 blocks -> 4,032 floats
    assert not ws.supports_ce(1345)        # pads to 1,408 rows -> 4,224 floats
    # widths: multiples of 8 up to 2,048; rows 16-byte aligned
    assert not ws.supports_rms(_Rows(64, 2056))
    assert not ws.supports_rms(_Rows(64, 768, ptr=4100))
    assert not ws.supports_qk(_Rows(64, 768), _Rows(64, 512))


def test_workspace_exchange_arguments_use_device_epochs():
    ws = _workspace(stat_rows=131072)
    ws.stat = ["even-slabs", "odd-slabs"]
    ws.base, ws.off_stat, ws.off_stat_flags = 1 << 20, [4096, 8192], 1024
    ws.stat_flags, ws.rank, ws.tp, ws.epoch_stat = "flags", 1, 2, 0
    ws._ctr, ws._done = [10, 11, 12], [20, 21, 22]
    kw = ws.exchange_kwargs()
    assert kw["epoch_ctr"] == 12 and kw["epoch_done"] == 22           # the statistics kind's counter
    assert kw["peer_recv"] == "even-slabs" and kw["peer_recv_odd"] == "odd-slabs"
    assert kw["my_recv"] == (1 << 20) + 4096 and kw["my_recv_odd"] == (1 << 20) + 8192
    assert "epoch" not in kw and ws._stat_kwargs()["epoch"] == 0 and ws.epoch_stat == 2
