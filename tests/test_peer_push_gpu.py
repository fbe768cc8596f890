"""matmul_peer_push, the C exchange kernel of the row-sharded multi-GPU GEMM (needs a B200).

On one GPU the "peer" buffers are other allocations on the same device: the
kernel only stores through the addresses it is given, so this checks its
indexing, its peer rotation and the C-ABI's argument checks; the 2- and 8-GPU
runs of bench.py check it across NVLink (an FP64 check of the exchanged rows).
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("peers,rows,ctas", [(1, 1, 0), (3, 37, 4), (7, 1000, 16), (7, 5, 64)])
def test_push_copies_the_block_to_every_destination(native, peers, rows, ctas):
    n = 132                                       # 528-byte rows: 16-byte multiples
    src_full = torch.randn((rows + 2, n), device="cuda")
    dsts = [torch.full((rows + 2, n), -7.0, device="cuda") for _ in range(peers)]
    lo, hi = 1, rows + 1                         # an interior block of rows
    row_bytes = n * 4
    native.peer_push(src_full.data_ptr() + lo * row_bytes, [d.data_ptr() + lo * row_bytes for d in dsts],
                     (hi - lo) * row_bytes, ctas=ctas)
    torch.cuda.synchronize()
    for d in dsts:
        assert torch.equal(d[lo:hi], src_full[lo:hi])
        assert torch.all(d[:lo] == -7.0) and torch.all(d[hi:] == -7.0)


def test_push_rejects_bad_arguments(native):
    a = torch.zeros(64, device="cuda")
    b = torch.zeros(64, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 16"):
        native.peer_push(a.data_ptr(), [b.data_ptr()], 20)
    with pytest.raises(RuntimeError, match="16-byte aligned"):
        native.peer_push(a.data_ptr() + 4, [b.data_ptr()], 16)
    with pytest.raises(RuntimeError, match="between 0 and 7"):
        native.peer_push(a.data_ptr(), [b.data_ptr()] * 8, 16)
    native.peer_push(a.data_ptr(), [], 16)        # nothing to do
