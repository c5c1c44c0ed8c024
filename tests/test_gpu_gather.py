"""The gathered-output path of the attention kernel (qflash_i8_fwd_gather) on
one GPU: the "peer" copy and the peer's signal words are buffers of the same
GPU, so the copies, the bulk stores and the barrier run without a second
process.  The barrier's wait is bounded: with a flag that nothing sets it
gives up, records bit 256 in the device error word and the context keeps
working."""
import pytest
import torch

pytestmark = pytest.mark.gpu

SIG_WORDS = 128
X_FLAG, X_VAL = 16, 64   # qflash_peer_max: flags and values in the signal words


def _case(Z, H, N, D, seed=0):
    from qflash_b200 import kernel as K
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(Z, H, N, D, device="cuda", generator=g) for _ in range(3))
    qs, ks, vs = K.tensor_scales(q, k, v)
    prm = K.fixed_point_params(float((qs * ks).item()), D, None)[1:]
    return tuple(K.quantize(t, s) for t, s in ((q, qs), (k, ks), (v, vs))), prm


def _launch(q8, k8, v8, o, prm, o_peers, barrier):
    from qflash_b200 import kernel as K
    K.launch_int8(q8, k8, v8, o, *prm, o_peers=o_peers, barrier=barrier)


@pytest.mark.parametrize("Z,H,N,D", [(3, 4, 197, 64), (2, 3, 49, 32), (2, 2, 100, 128), (1, 1, 5, 64),
                                     (2, 2, 70, 256)])
def test_gather_copies_equal_local_output(Z, H, N, D):
    """Every row lands in o and in each peer copy, for the bulk-copy layouts
    (dense rows, D <= 64) and the per-thread stores (D = 128, and D = 256,
    which runs as two launches with the barrier closing the second); the
    barrier passes when every rank's flag is set."""
    from qflash_b200 import _lib
    from qflash_b200 import kernel as K
    (q8, k8, v8), prm = _case(Z, H, N, D)
    ref = torch.empty_like(v8)
    K.launch_int8(q8, k8, v8, ref, *prm)
    o = torch.full_like(v8, 7)
    peers = [torch.full_like(v8, 9) for _ in range(2)]
    sig = torch.zeros(SIG_WORDS, dtype=torch.int32, device="cuda")
    sig_peers = [torch.zeros(SIG_WORDS, dtype=torch.int32, device="cuda") for _ in range(2)]
    sig[1] = 1
    sig[2] = 1      # the other two ranks of this launch have announced epoch 1 already
    _launch(q8, k8, v8, o, prm, [p.data_ptr() for p in peers],
            (sig.data_ptr(), [s.data_ptr() for s in sig_peers], 0, 1))
    torch.cuda.synchronize()
    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0
    assert torch.equal(o, ref)
    for p in peers:
        assert torch.equal(p, ref)
    assert int(sig[0]) == 1 and int(sig[8]) == 0                 # own flag set, CTA counter reset
    for s in sig_peers:
        assert int(s[0]) == 1                                     # this rank's flag in the peers' words


def test_gather_barrier_times_out_on_a_flag_nothing_sets():
    from qflash_b200 import _lib
    from qflash_b200 import kernel as K
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.device_error(stream) == 0
    (q8, k8, v8), prm = _case(2, 2, 64, 64, seed=1)
    ref = torch.empty_like(v8)
    K.launch_int8(q8, k8, v8, ref, *prm)
    o, peer = torch.empty_like(v8), torch.empty_like(v8)
    sig = torch.zeros(SIG_WORDS, dtype=torch.int32, device="cuda")
    sig_peer = torch.zeros(SIG_WORDS, dtype=torch.int32, device="cuda")
    # rank 1 of 2: rank 0's flag (sig[0]) is never written -> the wait gives up (~2 s)
    _launch(q8, k8, v8, o, prm, [peer.data_ptr()], (sig.data_ptr(), [sig_peer.data_ptr()], 1, 1))
    torch.cuda.synchronize()
    assert _lib.device_error(stream) == 256
    assert torch.equal(o, ref) and torch.equal(peer, ref)        # the rows were written before the wait
    # the context still works, and a later launch whose flags are set passes
    sig[0] = 2
    _launch(q8, k8, v8, o, prm, [peer.data_ptr()], (sig.data_ptr(), [sig_peer.data_ptr()], 1, 2))
    torch.cuda.synchronize()
    assert _lib.device_error(stream) == 0
    assert int(sig[1]) == 2 and int(sig_peer[1]) == 2


def test_gather_arguments_checked():
    from qflash_b200 import _lib
    from qflash_b200 import kernel as K
    (q8, k8, v8), prm = _case(1, 1, 32, 64)
    o = torch.empty_like(v8)
    peer = torch.empty(v8.numel() + 16, dtype=torch.int8, device="cuda")
    with pytest.raises(_lib.QFlashError, match="ALIGN"):          # different 16-byte phase from o
        _launch(q8, k8, v8, o, prm, [peer.data_ptr() + 1], None)
    sig = torch.zeros(SIG_WORDS, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.QFlashError, match="epoch"):          # epoch 0
        _launch(q8, k8, v8, o, prm, [peer.data_ptr()], (sig.data_ptr(), [sig.data_ptr()], 0, 0))
    with pytest.raises(_lib.QFlashError, match="rank"):           # rank outside [0, n_peers]
        _launch(q8, k8, v8, o, prm, [peer.data_ptr()], (sig.data_ptr(), [sig.data_ptr()], 2, 1))


def _peer_max(vals, sig, sig_peer, rank, epoch):
    from qflash_b200 import _lib
    out = torch.empty_like(vals)
    _lib.peer_max(vals, out, sig.data_ptr(), [sig_peer.data_ptr()], rank, epoch,
                  torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out


def test_peer_max_reduces_over_ranks_and_keeps_nan():
    from qflash_b200 import _lib
    stream = torch.cuda.current_stream().cuda_stream
    sig = torch.zeros(SIG_WORDS, dtype=torch.int32, device="cuda")
    sig_peer = torch.zeros(SIG_WORDS, dtype=torch.int32, device="cuda")
    for epoch, mine, theirs, want in ((1, [1.0, 7.0, 2.5], [3.0, -1.0, 2.5], [3.0, 7.0, 2.5]),
                                      (2, [0.5, float("nan"), 4.0], [0.25, 1.0, 8.0], [0.5, float("nan"), 8.0])):
        par = 8 * (epoch & 1)
        # rank 1 (the "peer") has written its values and flag into this rank's words
        sig.view(torch.float32)[X_VAL + 4 * (par + 1):X_VAL + 4 * (par + 1) + 3] = torch.tensor(theirs, device="cuda")
        sig[X_FLAG + 1] = epoch
        out = _peer_max(torch.tensor(mine, device="cuda"), sig, sig_peer, 0, epoch)
        assert _lib.device_error(stream) == 0
        assert torch.equal(out.isnan(), torch.tensor(want, device="cuda").isnan())
        assert torch.equal(out.nan_to_num(), torch.tensor(want, device="cuda").nan_to_num())
        # this rank's values and flag went into the peer's words
        got = sig_peer.view(torch.float32)[X_VAL + 4 * par:X_VAL + 4 * par + 3]
        assert torch.equal(got.nan_to_num(), torch.tensor(mine, device="cuda").nan_to_num())
        assert int(sig_peer[X_FLAG]) == epoch and int(sig[X_FLAG]) == epoch


def test_peer_max_times_out_on_a_flag_nothing_sets():
    from qflash_b200 import _lib
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.device_error(stream) == 0
    sig = torch.zeros(SIG_WORDS, dtype=torch.int32, device="cuda")
    sig_peer = torch.zeros(SIG_WORDS, dtype=torch.int32, device="cuda")
    out = _peer_max(torch.tensor([1.0, 2.0], device="cuda"), sig, sig_peer, 1, 1)   # rank 0 never announces
    assert _lib.device_error(stream) == 256
    assert bool(out.isnan().all())
    sig[X_FLAG] = 2
    sig.view(torch.float32)[X_VAL:X_VAL + 2] = torch.tensor([5.0, 0.0], device="cuda")
    out = _peer_max(torch.tensor([1.0, 2.0], device="cuda"), sig, sig_peer, 1, 2)
    assert _lib.device_error(stream) == 0
    assert out.tolist() == [5.0, 2.0]
