"""Host-side checks of the tuning options and of the switch API's argument
validation (no GPU: nothing here queues work)."""

import pytest
import torch

from aegaeon_b200 import _lib, switch


def test_set_option_accepts_known_names_and_rejects_others():
    lib = _lib.lib()
    assert lib.kvx_set_option(b"ce_streams", 2) == 0
    assert lib.kvx_set_option(b"ce_streams", 1) == 0
    assert lib.kvx_set_option(b"ce_max_copy", 256 << 20) == 0
    assert lib.kvx_set_option(b"ce_max_copy", 0) == 0
    assert lib.kvx_set_option(b"ce_min_run", 4 << 20) == 0
    for name in (b"sm_ctas_host", b"sm_ctas_host_out", b"sm_ctas_host_in"):
        assert lib.kvx_set_option(name, 96) == 0, name
        assert lib.kvx_set_option(name, 0) == 0, name  # back to the split by direction
    assert lib.kvx_set_option(b"ce_streams", 0) == _lib.KVX_ERR_INVALID_ARGUMENT
    assert lib.kvx_set_option(b"ce_streams", 9) == _lib.KVX_ERR_INVALID_ARGUMENT
    assert lib.kvx_set_option(b"ce_max_copy", -1) == _lib.KVX_ERR_INVALID_ARGUMENT
    for name, good, bad in ((b"bulk_waves", (1, 16), (0, 65)),
                            (b"bulk_ctas_per_sm", (1, 2), (0, 3)),
                            (b"vec_bytes", (16, 32), (8, 64)),
                            (b"staging_bulk", (0, 1), ()),
                            (b"host_bulk", (1, 0), ())):
        for v in good:
            assert lib.kvx_set_option(name, v) == 0, (name, v)
        for v in bad:
            assert lib.kvx_set_option(name, v) == _lib.KVX_ERR_INVALID_ARGUMENT, (name, v)
    # back to the defaults the other tests expect
    for name, v in ((b"bulk_waves", 16), (b"bulk_ctas_per_sm", 2), (b"vec_bytes", 32),
                    (b"staging_bulk", 1), (b"host_bulk", 0)):
        assert lib.kvx_set_option(name, v) == 0
    assert lib.kvx_set_option(b"no_such_knob", 1) == _lib.KVX_ERR_INVALID_ARGUMENT
    assert b"no_such_knob" in lib.kvx_last_error()
    assert lib.kvx_set_option(None, 1) == _lib.KVX_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _lib.set_option("no_such_knob", 1)


def test_upload_weights_validates_pairs_before_any_cuda_call():
    h = torch.zeros(16, dtype=torch.uint8)
    with pytest.raises(ValueError, match="device tensor, host tensor"):
        switch.upload_weights([(h.clone(), h)])
    switch.upload_weights([])  # nothing to do


def test_upload_weights_entry_point_checks_arguments():
    lib = _lib.lib()
    vp, u64 = _lib.ctypes.c_void_p, _lib.ctypes.c_uint64
    assert lib.kvx_upload_weights(None, None, None, 0, 1 << 20, 1, None) == 0
    assert lib.kvx_upload_weights(None, None, None, -1, 1 << 20, 1, None) == \
        _lib.KVX_ERR_INVALID_ARGUMENT
    assert lib.kvx_upload_weights(None, None, None, 1, 1 << 20, 1, None) == \
        _lib.KVX_ERR_INVALID_ARGUMENT
    one = (vp * 1)(0)
    size = (u64 * 1)(16)
    assert lib.kvx_upload_weights(one, one, size, 1, 0, 1, None) == _lib.KVX_ERR_INVALID_ARGUMENT
