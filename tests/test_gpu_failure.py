"""Failure detection without a GPU fault: the peer exchange's bounded wait is made to run out.

The exchange kernel (the decode step's one-shot all-reduce over peer memory) waits for every
source's flag with a %globaltimer limit. Here it runs as rank 0 of a loopback group whose
mailboxes all live on this GPU; the absent sources' flags are never set, so the wait runs out,
the kernel raises ERR_TIMEOUT and returns, and the host reports SPB_ECUDA (the reference's
SP_ECUDA, sp_status.h:19-56) with the detail in spb_last_error(). The device and a resident
session stay usable afterwards. No process dies and no kernel is left waiting."""
import time

import numpy as np
import pytest

import spb200
import spmodel
import xref

pytestmark = pytest.mark.gpu


def test_exchange_complete_when_all_arrive(spb, cuda_ok):
    for world in (2, 4, 8):
        assert spb.spb_tp_p2p_loopback(world, 0, 1000, 1000) == spb200.SPB_OK, spb.spb_last_error()


def test_exchange_wait_times_out_and_device_stays_usable(xr, spb, cuda_ok):
    cfg = spmodel.CONFIGS["micro_gemma"]
    T = spmodel.gen_model(cfg, seed=2)
    m = spb200.Model.upload(cfg, T)
    s = m.session(64)
    toks = spmodel.gen_tokens(3, 8, cfg.n_vocab)
    s.prefill(toks, logits=False)
    for world, absent in ((2, 0b10), (8, 0b10100000)):
        t0 = time.perf_counter()
        rc = spb.spb_tp_p2p_loopback(world, absent, 50, 256)
        dt = time.perf_counter() - t0
        assert rc == spb200.SPB_ECUDA
        assert b"timeout" in spb.spb_last_error()
        assert 0.05 <= dt < 5.0                       # the wait ran its 50 ms limit, then ended
    # the context, the device and the session all still work, byte-exact
    assert spb.spb_tp_p2p_loopback(4, 0, 1000, 64) == spb200.SPB_OK
    xs = xr.session(xref.build_desc(cfg, T), 64)
    xs.prefill(toks)
    tok = 5
    for _ in range(3):
        a, am = s.step_argmax(tok)
        assert np.array_equal(a.view(np.uint32), xs.step(tok).view(np.uint32))
        tok = am
    s.close()
    m.free()


def test_loopback_rejects_bad_args(spb, cuda_ok):
    assert spb.spb_tp_p2p_loopback(1, 0, 10, 8) == spb200.SPB_EBADARG      # no peer
    assert spb.spb_tp_p2p_loopback(2, 1, 10, 8) == spb200.SPB_EBADARG      # rank 0 itself absent
    assert spb.spb_tp_p2p_loopback(2, 4, 10, 8) == spb200.SPB_EBADARG      # a source beyond world
    assert spb.spb_tp_p2p_loopback(2, 0, 0, 8) == spb200.SPB_EBADARG       # no limit
