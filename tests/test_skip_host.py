"""Host logic of the synapse-skipping paths (no GPU): the flag bits the context manager
sets for a call, and the capacity checks that mirror the kernels' table builders."""
import torch

import ltc_cuda


def test_flag_bits_of_the_context_manager():
    base = ltc_cuda._call_flags_now()
    with ltc_cuda.skip_zero_synapses():
        assert ltc_cuda._call_flags_now() & ltc_cuda.LTC_FLAG_SKIP_ZERO_SYNAPSES
        assert not ltc_cuda._call_flags_now() & ltc_cuda.LTC_FLAG_SKIP_ZERO_SENSORY
        with ltc_cuda.skip_zero_synapses(sensory=True):
            assert ltc_cuda._call_flags_now() & ltc_cuda.LTC_FLAG_SKIP_ZERO_SENSORY
        with ltc_cuda.skip_zero_synapses(False, sensory=True):  # off turns both off
            assert not ltc_cuda._call_flags_now() & (ltc_cuda.LTC_FLAG_SKIP_ZERO_SYNAPSES |
                                                     ltc_cuda.LTC_FLAG_SKIP_ZERO_SENSORY)
        assert not ltc_cuda._call_flags_now() & ltc_cuda.LTC_FLAG_SKIP_ZERO_SENSORY
    assert ltc_cuda._call_flags_now() == base
    # the sensory bit lies above the lean segment-length field (bits 8..23)
    assert ltc_cuda.LTC_FLAG_SKIP_ZERO_SENSORY >> ltc_cuda.LTC_LEAN_CHUNK_SHIFT > 0xFFFF


def test_sensory_capacity_check():
    d, q = torch.arange(200)[:, None], torch.arange(64)[None, :]
    band = (((q - d) % 64) < 48).float()
    assert ltc_cuda.skip_zero_sensory_fits(band)           # 48 per input and per column in each chunk
    worse = band.clone()
    worse[130, (130 + 48) % 64] = 1.0                      # one input of the third chunk feeds 49
    assert not ltc_cuda.skip_zero_sensory_fits(worse)
    col = band.clone()
    col[70, :] = 0.0
    col[70, 5] = 1.0
    col[71, 5] = 1.0
    # column 5 in chunk 64..127: every input's band covers it except where removed
    assert ltc_cuda.skip_zero_sensory_fits(col) == (int(col[64:128, 5].sum()) <= 48)
    assert ltc_cuda.skip_zero_sensory_fits(torch.ones(300, 32))   # H <= 32: any pattern
    wide = (((torch.arange(512)[None, :] - torch.arange(300)[:, None]) % 64) < 40).float()
    assert ltc_cuda.skip_zero_sensory_fits(wide)                   # H > 64: per 64 x 64 block
    wide[7, 100:164] = 1.0                                          # 64 in one block row
    assert not ltc_cuda.skip_zero_sensory_fits(wide)
