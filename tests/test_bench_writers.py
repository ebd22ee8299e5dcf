"""CPU checks of the bench's file and writer workloads: the expert file it writes for the `file` config
opens through wexb_file_open, its record table matches what the bench reads offsets from, every record
reads back with its SHA-256, and the miss trace draws distinct experts of the rank's shard."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_file_config_workload(tmp_path, monkeypatch):
    sys.path.insert(0, ROOT)
    import bench
    import wexcuda
    monkeypatch.setenv('WEXB_FILE_DIR', str(tmp_path))
    cfg = dict(bench.CONFIGS['file'], hidden=1024, ffn=512, layers=2, experts=8, misses=6)
    for rank, world in ((0, 1), (1, 2)):
        path, owners, experts, blob = bench.write_expert_file(cfg, rank, world, 4)
        assert os.path.dirname(path) == str(tmp_path)
        assert all(e % world == rank for _, e in owners) and len(owners) == 2 * 8 // world
        offsets = bench.file_record_offsets(path)
        assert sorted(offsets) == sorted(owners)
        with open(path, 'rb') as fh:
            for e in experts:
                fh.seek(offsets[(e.layer, e.index)])
                assert fh.read(len(e.record)) == e.record
        f = wexcuda.ExpertFile(path)
        assert f.info()[:3] == (2, 8, len(owners))
        keys = bench.miss_keys(owners, cfg['misses'], 3)
        assert len(set(keys)) == len(keys) == min(cfg['misses'], len(owners))
        bad, status, got = f.read(keys, check=True)
        assert bad == 0 and got == sum(len(e.record) for e in experts if (e.layer, e.index) in set(keys))
        f.close()
        os.remove(path)


def test_encode_config_pool():
    sys.path.insert(0, ROOT)
    import bench
    import synth
    cfg = dict(bench.CONFIGS['encode'], hidden=1024, ffn=512, layers=2, experts=2)
    ex, blob = bench.encode_pool(cfg, 4)
    assert len(ex) == 4 and len(blob) == synth.MODEL_BYTES
    st, rec = synth.encode(blob, ex[0].entry, ex[0].coded, ex[0].flags, ex[0].owner)
    assert st == 0 and rec[:4] == b'WNR3'
