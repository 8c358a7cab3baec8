"""Peer-exchange primitives on one GPU: a signal followed by a wait in stream
order passes, and a wait on a flag that nothing sets gives up after its bound
(~2 s), records its code in the device error word and leaves the GPU usable.
No kernel waits on another running kernel here: the signal kernel completes
before the wait kernel starts."""
import pytest
import torch

from c_gpt2_b200 import ops, peer

pytestmark = pytest.mark.gpu


def test_signal_then_wait_passes(cuda):
    buf = peer.PeerBuffer(4096)
    try:
        peer.signal([buf.local], 7)
        peer.wait(buf.local, 1, 7)
        torch.cuda.synchronize()
        assert ops.device_error(reset=True) == 0
        assert int(peer.view(buf.local, (1,), torch.int32).item()) == 7
    finally:
        buf.close()


def test_wait_on_unset_flag_gives_up_and_reports(cuda):
    buf = peer.PeerBuffer(4096)
    try:
        peer.wait(buf.local + 64, 2, 1)  # two flags nothing ever sets
        torch.cuda.synchronize()
        assert ops.device_error(reset=True) == 0x1301
        x = torch.arange(8, device=cuda, dtype=torch.float32)
        assert float(x.sum().item()) == 28.0  # the context is still usable
    finally:
        buf.close()
