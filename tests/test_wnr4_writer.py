"""The WNR4 kind-MX writer of wex-wrn2_b200 (csrc/tools/wexb_wnr4.c: WNM4 training and the record
encoder) against the reference's own WNR4 decoder (oracle/_ref/wnr4_tools.so) and the oracle: every
record it writes decodes to the expected slab, for both position-bucket settings, canonical zero, the
ceil form, tile sizes G = 1, 4 and 32, and short last tiles."""
import ctypes

import pytest

import oracle
import synth

U32 = ctypes.c_uint32


def ref():
    L = oracle.ref_lib('wnr4_tools')
    if L is None:
        pytest.skip('reference WNR4 tools not built (make -C oracle ref)')
    return L


@pytest.mark.parametrize('hidden,ffn,pb,G,cz,mode', [(1024, 512, 1, 32, False, 0), (1024, 512, 5, 32, True, 0),
                                                     (256, 96, 1, 4, False, 2), (1024, 512, 5, 1, True, 3),
                                                     (2048, 768, 1, 32, True, 2)])
def test_reference_decoder_accepts_our_records(hidden, ffn, pb, G, cz, mode):
    R = ref()
    ex = [synth.Expert(hidden, ffn, 1, i, 9000 + 17 * i + hidden + G, 0.02, cz, mode, 0.03 if cz else 0.0)
          for i in range(3)]
    blob4 = synth.train_model4([(e.entry, e.coded) for e in ex[:2]], pb)
    mid = oracle.lib().oracle_wnm4_id(blob4, len(blob4))
    assert mid
    h = R.wnr4t_model_open(blob4, len(blob4))
    assert h
    for k, e in enumerate(ex):
        rec = synth.encode4(blob4, e.entry, e.coded, e.flags, 40 + k, G)
        assert rec is not None and len(rec) % 4096 == 0
        assert int.from_bytes(rec[4:8], 'little') == mid
        geo = synth.geo4(e.entry)
        out = ctypes.create_string_buffer(len(e.source))
        assert R.wnr4t_decode(h, (U32 * 13)(*geo), rec, len(rec), 40 + k, out, 1) == 0
        assert out.raw == e.expected
        err, slab = oracle.wnr4_decode(blob4, geo, rec, 40 + k, len(e.source))
        assert err == 0 and slab == e.expected
        # the wrong owner is refused by both
        assert R.wnr4t_decode(h, (U32 * 13)(*geo), rec, len(rec), 41 + k, out, 1) != 0
    R.wnr4t_model_close(h)


def test_incompressible_expert_is_not_written():
    e = synth.Expert(1024, 512, 0, 0, 5, 0.02, False, 1)
    blob4 = synth.train_model4([(synth.Expert(1024, 512, 0, 1, 6, 0.02).entry, synth.Expert(1024, 512, 0, 1, 6, 0.02).coded)])
    assert synth.encode4(blob4, e.entry, e.coded, e.flags, 0, 32) is None
