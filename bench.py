#!/usr/bin/env python3
"""Decode throughput of WEX4 expert records into HBM on B200 (decoded GB/s and experts/s).

Workload (default "large", the largest single-GPU configuration): MoE experts of hidden 7168 and expert
FFN 2048 (gate/up [2048 x 7168], down [7168 x 2048] in MXFP4: E2M1 nibbles packed two per byte, one E8M0
scale per 32), 58 layers x 192 experts, per-layer sigma drawn from U(0.01, 0.04), about 3 % of the zero
nibbles written as -0, encoded as WNR3 records in canonical-zero mode (value-exact; chunks 2048:512)
under one WNM2 model. A step is one token of routed decode: for each of the 58 layers the top-8 of a
Zipf(1.1) popularity over that layer's experts (seeded), i.e. 464 expert records of 23.4 MB, 10.9 GB of
decoded slabs. The routing trace has one token step, drawn once and used by every step (464 distinct
records, 9.9 GB of page-locked host memory a rank, so that eight ranks fit one host). Inputs are seeded
synthetic data (no dataset is involved) and larger than L2 between steps (the step's records are 80 x L2).

  value  records resident in HBM (wexb_resident_*), the step's records decoded by one persistent launch
         (scale, weight and commit work drained from one queue; two decodes queued, so the next step is
         planned while this one runs), timed with CUDA events on the launching stream; roofline: that
         launch against HBM (records read, slabs written, the error-gated commit) and, as
         roofline.issue, against the warp-instruction issue rate that binds it
  e2e    from pinned host memory through the C ABI: per layer one call of 8 records (H2D inside the
         timed region, statuses read back), 58 calls a step, timed by the host clock (max over ranks);
         the headline keeps --depth calls in flight (wexb_batch_submit / wexb_batch_wait), e2e.sync is
         the synchronous drop-in wex_cuda_decode_batch_to_device; each record decodes as its upload lands
  gpu_reference  the reference's own CUDA helper (compiled unchanged for sm_100a) on the same pinned
         records and destinations, the synchronous call (1 GPU)

N GPUs (torchrun): expert-parallel placement, rank r decodes the experts whose id = r mod N (weak
scaling: 464 records per rank per step); the only collectives are the max-over-ranks timing and a
final gather of per-rank outcome counters.

--impl reference: the reference's own CPU decoder (wex_nr2_decode via its wex_nr3_decode tool,
compiled from its sources into oracle/_ref) on all host cores, one record per core, on a bounded sample
of the same workload whose records the reference's own encoder made (nothing of this repository is
loaded in that process).

Other workloads (--config): mid (hidden 2048, FFN 768, 48 x 128, byte-exact), box (1,536 large experts
streamed by every step, each record's SHA-256 checked on the GPU before its decode may commit), wnr4
(draft codec 8 through the WNR4 ABI), tiny-file and mixed (WEX4 containers checked by wex4_check), file
(expert misses read from a container file on disk: wexb_file_decode) and encode (the GPU record writer).
"""
import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, 'wex-wrn2_b200'))
# One hardware work queue per stream (read when the CUDA context is made): the library's upload, metadata,
# kernel and hash-lane streams then never wait behind one another's long launches.
os.environ.setdefault('CUDA_DEVICE_MAX_CONNECTIONS', '32')

CONFIGS = {
    'tiny': dict(hidden=1024, ffn=512, layers=1, experts=8, batch=8, cz=False, sigma=(0.02, 0.02), neg_zero=0.0),
    'mid': dict(hidden=2048, ffn=768, layers=48, experts=128, batch=8, cz=False, sigma=(0.01, 0.04), neg_zero=0.0),
    # the largest single-GPU workload (the default): a token step routes 464 experts of 23.4 MB; the routing
    # trace has `trace_steps` distinct token steps, cycled, so that the distinct records fit in host memory
    # with eight ranks on one host (9.9 GB of page-locked records a rank; the records of a step are 80 x L2)
    'large': dict(hidden=7168, ffn=2048, layers=58, experts=192, batch=8, cz=True, sigma=(0.01, 0.04), neg_zero=0.03,
                  lean=True, trace_steps=1),
    # whole-box streaming: 1536 large experts, each rank decodes all of its shard every step
    'box': dict(hidden=7168, ffn=2048, layers=8, experts=192, batch=8, cz=True, sigma=(0.01, 0.04), neg_zero=0.03,
                lean=True, all_experts=True, verify=True),
    # WNR4 kind MX (draft codec 8) through the ABI 5: large experts, G = 32, one batch call per layer
    'wnr4': dict(hidden=7168, ffn=2048, layers=2, experts=8, batch=8, cz=True, sigma=(0.01, 0.04), neg_zero=0.03,
                 wnr4=True),
    # containers: a WEX4 file per rank, checked and decoded by wex4_check (per-record SHA-256 against
    # the index, codec dispatch, decode); tiny = the 8 experts plus one RAW expert, mixed = one routed
    # step of large experts, 10 % uniform-random (stored RAW), 30 % WNR4 kind MX, the rest WNR3 CZ
    'tiny-file': dict(hidden=1024, ffn=512, layers=1, experts=9, batch=9, cz=False, sigma=(0.02, 0.02), neg_zero=0.0,
                      container=True, raw=(8,), wnr4_frac=0.0),
    'mixed': dict(hidden=7168, ffn=2048, layers=58, experts=192, batch=8, cz=True, sigma=(0.01, 0.04), neg_zero=0.03,
                  container=True, raw_frac=0.10, wnr4_frac=0.30),
    # expert misses served from a container file: every step reads `misses` distinct experts of the rank's
    # file (a seeded permutation, as bench/wex_io.c draws them) and decodes them into HBM (wexb_file_*)
    'file': dict(hidden=2048, ffn=768, layers=8, experts=128, batch=8, cz=False, sigma=(0.01, 0.04), neg_zero=0.0,
                 file=True, misses=256),
    # the writer side: 64 coded mid experts counted (model training) and encoded as WNR3 records per step
    'encode': dict(hidden=2048, ffn=768, layers=8, experts=8, batch=64, cz=True, sigma=(0.01, 0.04), neg_zero=0.03,
                   encode=True),
}
SEED = 20261201
MEASURED_PEAKS = os.path.join(ROOT, 'MEASURED_PEAKS.json')


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---- workload -------------------------------------------------------------------------------------
def layer_sigmas(cfg):
    rng = np.random.default_rng(SEED)
    lo, hi = cfg['sigma']
    return rng.uniform(lo, hi, cfg['layers'])


def routing_trace(cfg, steps, rank, world, layers):
    """[step][layer] -> 8 distinct expert ids of this rank's shard (id % world == rank), Zipf(1.1); for a
    streaming config (all_experts) every expert of the shard, every step. A config with `trace_steps`
    draws that many token steps and cycles them."""
    shard = np.arange(rank, cfg['experts'], world)
    if cfg.get('all_experts'):
        return [[[int(e) for e in shard] for _ in range(layers)] for _ in range(steps)]
    period = cfg.get('trace_steps')
    if period and steps > period:
        base = routing_trace(cfg, period, rank, world, layers)
        return [base[s % period] for s in range(steps)]
    trace = []
    for layer in range(layers):
        rng = np.random.default_rng([SEED, layer, rank])
        order = rng.permutation(shard)                         # popularity rank of each expert
        p = 1.0 / np.arange(1, len(order) + 1) ** 1.1
        p /= p.sum()
        k = min(cfg['batch'], len(order))
        trace.append([list(rng.choice(order, size=k, replace=False, p=p)) for _ in range(steps)])
    return [[trace[l][s] for l in range(layers)] for s in range(steps)]


def build_pool(cfg, owners, threads, device=None):
    """WNM2 model (trained on one fixed expert per layer, the same on every rank) and the records. With a
    device and a lean config, the records are encoded by this library's GPU writer (wexb_encode_batch,
    byte-identical to the CPU encoder): the host threads only make the coded slabs."""
    import synth
    sig = layer_sigmas(cfg)
    train = [(l, l % cfg['experts']) for l in range(cfg['layers'])]
    blob, _ = synth.make_experts(cfg['hidden'], cfg['ffn'], train, seed=SEED, sigma=lambda l: sig[l], cz=cfg['cz'],
                                 neg_zero=cfg['neg_zero'], train_every=1, threads=threads)
    if device is not None and cfg.get('lean'):
        return blob, gpu_encoded_pool(cfg, owners, threads, blob, device)
    _, experts = synth.make_experts(cfg['hidden'], cfg['ffn'], owners, seed=SEED, sigma=lambda l: sig[l], cz=cfg['cz'],
                                    neg_zero=cfg['neg_zero'], threads=threads, blob=blob, lean=cfg.get('lean', False))
    return blob, experts


def gpu_encoded_pool(cfg, owners, threads, blob, device):
    """Lean experts (entry, record, .raw, .expected_sha) of the owners: host threads make each group's coded
    slabs (the same seeds as synth.make_experts) while the GPU encodes the previous group."""
    import synth
    import wexcuda
    sig = layer_sigmas(cfg)
    group = max(8, threads)

    def make(o):
        layer, idx = o
        e = synth.Expert(cfg['hidden'], cfg['ffn'], layer, idx, SEED * 1000003 + layer * 4099 + idx, sig[layer],
                         cfg['cz'], 0, cfg['neg_zero'])
        e.raw = len(e.source)
        e.expected_sha = hashlib.sha256(e.expected).digest()
        e.expected = None   # only its digest is kept (host memory: a rank holds its records and little else)
        return e
    out = []
    with ThreadPoolExecutor(threads) as pool, ThreadPoolExecutor(1) as ahead:
        pending = ahead.submit(lambda g: list(pool.map(make, g)), owners[:group])
        for at in range(0, len(owners), group):
            ex = pending.result()
            if at + group < len(owners):
                pending = ahead.submit(lambda g: list(pool.map(make, g)), owners[at + group:at + 2 * group])
            res = wexcuda.encode_batch(blob, [e.entry for e in ex], [e.coded for e in ex], [e.flags for e in ex],
                                       [e.owner for e in ex], True, 2048, 512, device)
            for e, (st, rec, _, _) in zip(ex, res):
                assert st in (0, 1), f'GPU encoder status {st}'
                if st == 0:
                    e.record, e.codec = rec, synth.CODEC_WNR3
                else:   # not smaller than raw: stored RAW with the source bytes (c/tools/wex_nr3_tools.c:85-103)
                    e.record = e.source + bytes(((e.raw + 4095) & ~4095) - e.raw)
                    e.codec = synth.CODEC_RAW
                    e.expected_sha = hashlib.sha256(e.source).digest()
                e.entry = synth.entry_with(e.entry, total=len(e.record), codec=e.codec)
                e.source = e.coded = e.expected = None
            pin_group(ex)
            out.extend(ex)
    return out


PINNED = []   # page-locked record buffers, kept for the life of the process


def pin_group(experts):
    """Moves the experts' records into one new page-locked buffer (each e.record becomes a view of it), so
    that a rank never holds a record twice in host memory."""
    import wexcuda
    buf = np.empty(sum(len(e.record) for e in experts), np.uint8)
    at = 0
    for e in experts:
        n = len(e.record)
        buf[at:at + n] = np.frombuffer(e.record, np.uint8)
        e.record = buf[at:at + n]
        at += n
    assert wexcuda.host_register(buf) == 0
    PINNED.append(buf)


def pinned_records(experts):
    """Every record in page-locked host memory (moved there unless it already is); returns (None, views)."""
    loose = [e for e in experts if not isinstance(e.record, np.ndarray)]
    for at in range(0, len(loose), 64):
        pin_group(loose[at:at + 64])
    return None, [e.record for e in experts]


def rec_arg(record):
    """A record (bytes or a page-locked view) as a ctypes pointer argument."""
    return record.ctypes.data if isinstance(record, np.ndarray) else record


# ---- clocks -------------------------------------------------------------------------------------
class Clocks:
    """nvidia-smi samples (200 ms) of this rank's GPU during the timed regions."""
    FIELDS = 'index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,' \
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,' \
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap'

    def __init__(self, gpu):
        self.gpu, self.proc, self.lines = gpu, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(self.gpu), f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=lambda: self.lines.extend(self.proc.stdout), daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable']}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.reader.join(timeout=5)
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.lines:
            f = [x.strip() for x in line.split(',')]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1])); mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith('active'):
                    reasons.add(n)
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': mx, 'reasons': sorted(reasons),
                'samples': len(sm)}


# ---- distributed plumbing ----------------------------------------------------------------------------
def dist_init():
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        os.environ.setdefault('NCCL_DEBUG', 'WARN')   # rank 0's stdout carries only the JSON line
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=torch.device('cuda', local))
    return world, rank, local


def _reduce_device():
    """Device of the reduction tensors: CUDA under NCCL, the host under gloo (the CPU rank tests)."""
    import torch.distributed as dist
    return 'cuda' if dist.get_backend() == 'nccl' else 'cpu'


def bind_to_gpu_numa_node(local):
    """Run this rank on the CPUs of its GPU's NUMA node, so that the pinned host records it allocates
    and fills (first touch) are local to the GPU's PCIe root. Returns the node, or None when the
    topology is not visible."""
    import torch
    try:
        props = torch.cuda.get_device_properties(local)
        bus = f'{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0'
        node = int(open(f'/sys/bus/pci/devices/{bus}/numa_node').read())
        if node < 0:
            return None
        cpus = set()
        for part in open(f'/sys/devices/system/node/node{node}/cpulist').read().strip().split(','):
            lo, _, hi = part.partition('-')
            cpus.update(range(int(lo), int(hi or lo) + 1))
        os.sched_setaffinity(0, cpus)
        return node
    except (OSError, ValueError, AttributeError):
        return None


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=_reduce_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def min_over_ranks(x, world):
    return -max_over_ranks(-x, world)


def sum_over_ranks(vals, world):
    if world == 1:
        return vals
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device=_reduce_device())
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [float(v) for v in t.tolist()]


def gather_outcomes(rows, world):
    """The per-record outcome table of every rank, on every rank (one all-gather after the run)."""
    if world == 1:
        return list(rows)
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, list(rows))
    return [r for part in out for r in part]


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---- CPU decoder of the reference (the baseline / the reference arm) -------------------------------
def reference_decode_rate(experts, blob, cores, min_seconds=10.0, max_records=None):
    """Decode records with the reference's CPU decoder (oracle/_ref/wex_nr3_tools.so: wex_nr3_decode ->
    wex_decode_nr2_record -> wex_nr2_decode), one record per host thread, until min_seconds of work.
    Returns (seconds, records decoded, decoded bytes, kind, sample description)."""
    sys.path.insert(0, os.path.join(ROOT, 'oracle'))
    import ctypes
    import oracle
    L = oracle.ref_lib('wex_nr3_tools')
    if L is None:
        raise RuntimeError('oracle/_ref/wex_nr3_tools.so is missing: build it with `make -C oracle ref`')
    sample = [e for e in experts if e.codec == 5][: (max_records or len(experts))]
    outs = [ctypes.create_string_buffer(e.raw) for e in sample[:cores]]

    def one(i):
        e = sample[i % len(sample)]
        st = L.wex_nr3_decode(blob, e.entry, rec_arg(e.record), e.layer, e.index, outs[i % cores])
        if st != 0:
            raise RuntimeError('reference decoder refused a record')
        return e.raw
    with ThreadPoolExecutor(cores) as pool:
        t0 = time.perf_counter()
        done, nbytes, n = 0, 0, 0
        while True:
            batch = list(pool.map(one, range(n, n + cores)))
            n += cores
            nbytes += sum(batch)
            done = n
            if time.perf_counter() - t0 >= min_seconds:
                break
        dt = time.perf_counter() - t0
    return dt, done, nbytes


def reference_file_rate(data, cores, min_seconds=10.0, lib='wex4_tools_ref'):
    """Check and decode the records of a WEX4 file with the reference's CPU tools, one record per host
    thread, until min_seconds of work: wex4_decode_record_buf of oracle/_ref/<lib>.so (SHA-256 against
    the index, then RAW / WNR3 / WBP1 decode; wex4_tools_fast.so is its fast WNR3 decoder), and for
    codec-8 records the SHA-256 then the reference WNR4 decoder (oracle/_ref/wnr4_tools.so).
    Returns (seconds, records, decoded bytes)."""
    sys.path.insert(0, os.path.join(ROOT, 'oracle'))
    import ctypes
    import oracle
    import synth
    L, W = oracle.ref_lib(lib), oracle.ref_lib('wnr4_tools')
    if L is None or W is None:
        raise RuntimeError(f'oracle/_ref/{lib}.so or wnr4_tools.so is missing: build them with `make -C oracle ref`')
    f = oracle.Wex4File(data)
    blobs = [f.blob(i) for i in range(len(f.blobs))]
    handles = {i: W.wnr4t_model_open(b, len(b)) for i, b in enumerate(blobs) if f.blobs[i]['kind'] == 3}
    geos = {}
    for r, rec in enumerate(f.records):
        if rec['codec'] == 8:
            ts = f.tensors[rec['first']:rec['first'] + 6]
            g = [0] * 13
            for m in range(3):
                g[1 + m], g[4 + m] = ts[m]['shape'][0] * ts[m]['shape'][1], ts[m]['shape'][1]
                g[7 + m], g[10 + m] = ts[m]['offset'], ts[3 + m]['offset']
            geos[r] = (ctypes.c_uint32 * 13)(*g)
    outs = [ctypes.create_string_buffer(f.max_decoded) for _ in range(cores)]

    def one(i):
        r = i % len(f.records)
        rec, out = f.records[r], outs[i % cores]
        stored = f.stored(r)
        if rec['codec'] == 8:
            if hashlib.sha256(stored).digest() != rec['sha']:
                raise RuntimeError('record hash differs')
            st = W.wnr4t_decode(handles[rec['blob'] - 1], geos[r], stored, len(stored), r, out, 1)
        else:
            blob = blobs[rec['blob'] - 1] if rec['blob'] else None
            st = L.wex4_decode_record_buf(f.page, f.file_bytes, f.index, len(f.index), r, stored, blob, 1, out)
        if st != 0:
            raise RuntimeError(f'reference refused record {r}: {st}')
        return rec['decoded']
    with ThreadPoolExecutor(cores) as pool:
        t0 = time.perf_counter()
        n, nbytes = 0, 0
        while True:
            nbytes += sum(pool.map(one, range(n, n + cores)))
            n += cores
            if time.perf_counter() - t0 >= min_seconds:
                break
        dt = time.perf_counter() - t0
    for h in handles.values():
        W.wnr4t_model_close(h)
    return dt, n, nbytes


# ---- the two arms ---------------------------------------------------------------------------------
def run_reference_container(args, cfg):
    """The reference arm of a container config: rank 0's file checked and decoded record by record by the
    reference's CPU tools on all host cores (a bounded sample of records per step)."""
    cores = os.cpu_count() or 1
    layers = args.layers or cfg['layers']
    owners = container_owners(cfg, 0, int(os.environ.get('WORLD_SIZE', '1')), layers)
    data, decoded, counts, _, _ = build_container(cfg, owners, cores)
    times = []
    for s in range(args.warmup + args.steps):
        dt, n, nb = reference_file_rate(data, cores, min_seconds=max(1.0, args.cpu_seconds / (args.warmup + args.steps)))
        if s >= args.warmup:
            times.append((dt, n, nb))
    total = sum(t[0] for t in times)
    nbytes, nrec = sum(t[2] for t in times), sum(t[1] for t in times)
    value = nbytes / total / 1e9
    print(json.dumps({
        'impl': 'reference', 'metric': 'decoded MXFP4 expert GB/s into HBM', 'value': round(value, 4), 'unit': 'GB/s',
        'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(1e3 * total / args.steps, 3),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'experts_per_s': round(nrec / total, 2),
        'config': {'workload': f'{args.config}: WEX4 container of {len(owners)} expert records, codecs {counts}'},
        'cpu_baseline': {'value': round(value, 4), 'unit': 'GB/s', 'cores': cores, 'kind': 'reference',
                         'sample': 'records of the file, one per host thread, the reference tool (SHA-256, decode)'},
        'e2e': {'value': round(value, 4), 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}))
    return 0


def run_reference_wnr4(args, cfg):
    """The reference arm of the wnr4 config: the reference's CPU WNR4 decoder (oracle/_ref/wnr4_tools.so,
    wnr4t_decode) on the same records, one record per host thread, all cores."""
    import ctypes
    import synth
    sys.path.insert(0, os.path.join(ROOT, 'oracle'))
    import oracle
    W = oracle.ref_lib('wnr4_tools')
    if W is None:
        print(json.dumps({'impl': 'reference', 'unavailable': 'oracle/_ref/wnr4_tools.so was not built'}))
        return 0
    cores = os.cpu_count() or 1
    sig = layer_sigmas(cfg)
    owners = [(l, i) for l in range(cfg['layers']) for i in range(cfg['batch'])]
    with ThreadPoolExecutor(cores) as pool:
        ex = list(pool.map(lambda o: synth.Expert(cfg['hidden'], cfg['ffn'], o[0], o[1], SEED * 31 + o[0] * 4099 + o[1],
                                                  sig[o[0]], cfg['cz'], 0, cfg['neg_zero']), owners))
        blob4 = synth.train_model4([(e.entry, e.coded) for e in ex[:4]])
        recs = list(pool.map(lambda k: synth.encode4(blob4, ex[k].entry, ex[k].coded, ex[k].flags, k, 32), range(len(ex))))
    geo = (ctypes.c_uint32 * 13)(*synth.geo4(ex[0].entry))
    raw = len(ex[0].source)
    h = W.wnr4t_model_open(blob4, len(blob4))
    outs = [ctypes.create_string_buffer(raw) for _ in range(cores)]

    def one(i):
        k = i % len(recs)
        if W.wnr4t_decode(h, geo, recs[k], len(recs[k]), k, outs[i % cores], 1) != 0:
            raise RuntimeError('reference WNR4 decoder refused a record')
        return raw
    times = []
    with ThreadPoolExecutor(cores) as pool:
        for s in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            nb = sum(pool.map(one, range(s * cores, (s + 1) * cores)))
            if s >= args.warmup:
                times.append((time.perf_counter() - t0, nb))
    W.wnr4t_model_close(h)
    total = sum(t for t, _ in times)
    value = sum(b for _, b in times) / total / 1e9
    print(json.dumps({
        'impl': 'reference', 'metric': 'decoded MXFP4 expert GB/s into HBM', 'value': round(value, 4), 'unit': 'GB/s',
        'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(1e3 * total / args.steps, 3),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'experts_per_s': round(cores * args.steps / total, 2),
        'config': {'workload': f'wnr4: WNR4 kind-MX records of hidden {cfg["hidden"]}, FFN {cfg["ffn"]}'},
        'cpu_baseline': {'value': round(value, 4), 'unit': 'GB/s', 'cores': cores, 'kind': 'reference',
                         'sample': f'{cores} records per step, one per host thread, reference wnr4t_decode'},
        'e2e': {'value': round(value, 4), 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}))
    return 0


def numpy_expert_slab(hidden, ffn, seed, sigma, neg_zero):
    """A seeded synthetic MXFP4 expert slab made with numpy alone, for the reference arm (whose process maps
    none of this repository's libraries): per matrix N(0, sigma) elements in blocks of 32, an E8M0 scale of
    floor(log2 amax) - 2, E2M1 codes {0, .5, 1, 1.5, 2, 3, 4, 6} by nearest with ties to the even code, the
    sign only on non-zero codes, and a fraction neg_zero of the zero codes written as -0. Layout: the
    scales of w1, w2, w3, then their packed nibbles (even element in the low nibble)."""
    rng = np.random.default_rng(seed)
    scales, packed = [], []
    for r, c in ((ffn, hidden), (hidden, ffn), (ffn, hidden)):
        g = rng.standard_normal((r * c // 32, 32), dtype=np.float32) * np.float32(sigma)
        amax = np.abs(g).max(axis=1)
        _, ex = np.frexp(amax)                      # amax = m 2^ex, m in [0.5, 1): floor(log2 amax) = ex - 1
        e = np.where(amax > 0, ex - 3, -127).clip(-127, 127).astype(np.int32)
        x = np.ldexp(g, -e[:, None])                # a power-of-two scaling: exact
        mag = np.minimum(np.abs(x), np.float32(6.0))
        code = ((mag > 0.25).astype(np.uint8) + (mag >= 0.75) + (mag > 1.25) + (mag >= 1.75) + (mag > 2.5) +
                (mag >= 3.5) + (mag > 5.0)).astype(np.uint8)
        nib = code | np.where((x < 0) & (code > 0), 8, 0).astype(np.uint8)
        if neg_zero:
            nib[(nib == 0) & (rng.random(nib.shape, dtype=np.float32) < neg_zero)] = 8
        scales.append((e + 127).astype(np.uint8).tobytes())
        packed.append((nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8).tobytes())
    return b''.join(scales) + b''.join(packed)


class RefExpert:
    """One record of the reference arm's pool."""
    def __init__(self, layer, index, entry, record, raw):
        self.layer, self.index, self.entry, self.record, self.raw = layer, index, entry, record, raw


def reference_pool(cfg, owners, cores):
    """The reference arm's inputs, made entirely by the reference's own tools (oracle/_ref/wex_nr3_tools.so,
    c/tools/wex_nr3_tools.c:37-120): numpy MXFP4 slabs, the coded domain (wex_nr3_prepare: canonical zero and
    ceil form), a WNM2 model trained on them (wex_nr3_count_expert, wex_nr3_build_model) and their WNR3
    records (wex_nr3_encode_record, chunks 2048:512). Returns (blob, experts) or None when the tools are
    not built."""
    import ctypes
    import synth   # pure Python here: expert_entry / entry_with load no library
    sys.path.insert(0, os.path.join(ROOT, 'oracle'))
    import oracle
    L = oracle.ref_lib('wex_nr3_tools')
    if L is None:
        return None
    sig = layer_sigmas(cfg)
    entry = synth.expert_entry(cfg['hidden'], cfg['ffn'])
    raw = synth.raw_bytes(cfg['hidden'], cfg['ffn'])

    def coded_of(o):
        layer, idx = o
        slab = numpy_expert_slab(cfg['hidden'], cfg['ffn'], [SEED, 7, layer, idx], sig[layer], cfg['neg_zero'])
        coded = ctypes.create_string_buffer(raw)
        flags = L.wex_nr3_prepare(entry, slab, 1 if cfg['cz'] else 0, coded, None)
        if flags < 0:
            raise RuntimeError('reference prepare refused an expert')
        return flags, coded
    with ThreadPoolExecutor(cores) as pool:
        coded = list(pool.map(coded_of, owners))
    wc, sc = np.zeros(3 * 567 * 16, np.uint64), np.zeros(3 * 256, np.uint64)
    for _, c in coded:
        if L.wex_nr3_count_expert(entry, c, wc.ctypes.data, sc.ctypes.data) != 0:
            raise RuntimeError('reference counts refused an expert')
    blob = ctypes.create_string_buffer(59408)
    if L.wex_nr3_build_model(wc.ctypes.data, sc.ctypes.data, blob, None) != 0:
        raise RuntimeError('reference model build failed')
    blob = blob.raw

    def encode(i):
        (layer, idx), (flags, c) = owners[i], coded[i]
        cap = 2 * raw + 65536
        out, used, total = ctypes.create_string_buffer(cap), ctypes.c_size_t(), ctypes.c_size_t()
        if L.wex_nr3_encode_record(blob, entry, c, flags, layer << 16 | idx, 2048, 512, out, cap, ctypes.byref(used),
                                   ctypes.byref(total)) != 0:
            raise RuntimeError('reference encoder did not compress an expert')
        rec = out.raw[:total.value]
        return RefExpert(layer, idx, synth.entry_with(entry, total=len(rec), codec=5), rec, raw)
    with ThreadPoolExecutor(cores) as pool:
        return blob, list(pool.map(encode, range(len(owners))))


def run_reference(args, cfg):
    world, rank, local = int(os.environ.get('WORLD_SIZE', '1')), int(os.environ.get('RANK', '0')), 0
    if rank != 0:
        return 0
    if cfg.get('container'):
        return run_reference_container(args, cfg)
    if cfg.get('wnr4'):
        return run_reference_wnr4(args, cfg)
    if cfg.get('file'):
        return run_reference_file(args, cfg)
    if cfg.get('encode'):
        return run_reference_encode(args, cfg)
    cores = os.cpu_count() or 1
    layers = args.layers or cfg['layers']
    trace = routing_trace(cfg, 1, 0, 1, layers)
    k = sum(len(trace[0][l]) for l in range(layers))   # records per step of the GPU arm's workload
    # the bounded sample decoded every step: the first ceil(cores / batch) layer batches of the first token
    # step, one record per host thread
    per_step = max(1, min(layers, -(-cores // cfg['batch'])))
    owners = [(l, int(e)) for l in range(per_step) for e in trace[0][l][:cfg['batch']]]
    t0 = time.time()
    made = reference_pool(cfg, owners, cores)
    if made is None:
        print(json.dumps({'impl': 'reference', 'unavailable': 'oracle/_ref/wex_nr3_tools.so was not built'}))
        return 0
    blob, experts = made
    log(f'[reference] {len(experts)} records made by the reference tools in {time.time() - t0:.1f} s')
    sys.path.insert(0, os.path.join(ROOT, 'oracle'))
    import ctypes
    import oracle
    L = oracle.ref_lib('wex_nr3_tools')
    outs = [ctypes.create_string_buffer(experts[0].raw) for _ in experts]

    def one(i):
        e = experts[i]
        if L.wex_nr3_decode(blob, e.entry, e.record, e.layer, e.index, outs[i]) != 0:
            raise RuntimeError('reference decoder refused a record')
        return e.raw
    times, nbytes, nrec = [], 0, 0
    with ThreadPoolExecutor(cores) as pool:
        for s in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            b = sum(pool.map(one, range(len(experts))))
            dt = time.perf_counter() - t0
            if s >= args.warmup:
                times.append(dt); nbytes += b; nrec += len(experts)
    total = sum(times)
    value = nbytes / total / 1e9
    line = {
        'impl': 'reference', 'metric': 'decoded MXFP4 expert GB/s into HBM', 'value': round(value, 4), 'unit': 'GB/s',
        'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(1e3 * total / args.steps, 3),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'experts_per_s': round(nrec / total, 2),
        'config': config_desc(args, cfg, k),
        'cpu_baseline': {'value': round(value, 4), 'unit': 'GB/s', 'cores': cores, 'kind': 'reference',
                         'sample': f'{len(experts)} records ({per_step} layer batch(es) of {cfg["batch"]} of the first '
                                   f'token step) decoded every step, one record per host thread, by the reference '
                                   f'wex_nr3_decode -> wex_nr2_decode; records made by the reference encoder'},
        'e2e': {'value': round(value, 4), 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line))
    return 0


# ---- WNR4 kind MX through its ABI ---------------------------------------------------------------------
def run_wnr4(args, cfg):
    """Every step decodes all experts of the config (layers x batch), one wnr4_cuda_decode_batch call of
    `batch` records per layer, from pinned host memory into HBM (H2D inside the timed region)."""
    import ctypes
    import torch
    import synth
    import wexcuda
    world, rank, local = dist_init()
    torch.cuda.set_device(local)
    U32, SZ, P, I = ctypes.c_uint32, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int
    W = wexcuda.lib()
    W.wnr4_cuda_register_model.argtypes = [P, SZ, I]
    W.wnr4_cuda_batch_submit.argtypes = [I, P, P, P, P, U32, I, P, P, P]
    W.wnr4_cuda_batch_wait.argtypes = [I, P]
    sig = layer_sigmas(cfg)
    owners = [(l, rank + world * i) for l in range(cfg['layers']) for i in range(cfg['batch'])]
    threads = max(1, (os.cpu_count() or 8) // max(1, int(os.environ.get('LOCAL_WORLD_SIZE', world))))
    t0 = time.time()
    with ThreadPoolExecutor(threads) as pool:
        ex = list(pool.map(lambda o: synth.Expert(cfg['hidden'], cfg['ffn'], o[0], o[1], SEED * 31 + o[0] * 4099 + o[1],
                                                  sig[o[0]], cfg['cz'], 0, cfg['neg_zero']), owners))
        blob4 = synth.train_model4([(e.entry, e.coded) for e in ex[:4]])
        recs = list(pool.map(lambda k: synth.encode4(blob4, ex[k].entry, ex[k].coded, ex[k].flags, k, 32), range(len(ex))))
    log(f'[rank {rank}] {len(ex)} WNR4 records encoded in {time.time() - t0:.1f} s')
    assert all(r is not None for r in recs)
    mid = int.from_bytes(recs[0][4:8], 'little')
    assert W.wnr4_cuda_register_model(blob4, len(blob4), local) == 0
    host, at = np.empty(sum(len(r) for r in recs), np.uint8), 0
    views = []
    for r in recs:
        host[at:at + len(r)] = np.frombuffer(r, np.uint8)
        views.append(host[at:at + len(r)])
        at += len(r)
    assert wexcuda.host_register(host) == 0
    raw = len(ex[0].source)
    expected = [hashlib.sha256(e.expected).digest() for e in ex]
    del ex
    k = len(recs)
    dst = torch.empty((2, k, raw), dtype=torch.uint8, device='cuda')   # steps alternate between two sets
    entry = synth.expert_entry(cfg['hidden'], cfg['ffn'])
    soff = [int.from_bytes(entry[44 + 4 * m:48 + 4 * m], 'little') for m in range(3)]
    woff = [int.from_bytes(entry[56 + 4 * m:60 + 4 * m], 'little') for m in range(3)]
    B = cfg['batch']
    geo = (U32 * 13)(*synth.geo4(entry))
    calls = [[], []]
    for half in (0, 1):
        base = dst[half].data_ptr()
        for c in range(0, k, B):
            sel = range(c, min(k, c + B))
            calls[half].append((len(sel), wexcuda._ptrs([views[i].ctypes.data for i in sel]),
                                (SZ * len(sel))(*[len(recs[i]) for i in sel]), (U32 * len(sel))(*sel),
                                wexcuda._ptrs([base + j * raw + soff[m] for j in sel for m in range(3)]),
                                wexcuda._ptrs([base + j * raw + woff[m] for j in sel for m in range(3)])))
    depth = 4   # the ABI's batches in flight per thread and device (WNR4_CUDA_SLOTS)

    def run(first, count):
        """Steps [first, first + count): every call submitted in order, each on its ticket's own stream,
        at most `depth` in flight, the oldest waited for before the next is submitted."""
        flight = []

        def wait_oldest():
            n, t = flight.pop(0)
            st = (ctypes.c_int * n)()
            assert W.wnr4_cuda_batch_wait(t, st) == 0, list(st)
        for s in range(first, first + count):
            for n, rp, tp, op, sp, wp in calls[s % 2]:
                if len(flight) == depth:
                    wait_oldest()
                t = W.wnr4_cuda_batch_submit(n, geo, rp, tp, op, mid, local, sp, wp, None)
                assert t >= 0, t
                flight.append((n, t))
        while flight:
            wait_oldest()
    run(0, args.warmup)
    h2d_gbs = measure_h2d(torch)
    clocks = Clocks(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()   # the calls use their own streams: host clock around the whole run
    run(args.warmup, args.steps)
    torch.cuda.synchronize()
    ms = max_over_ranks(1e3 * (time.perf_counter() - t0), world)
    barrier(world)
    clk = clocks.stop()
    last = (args.warmup + args.steps - 1) % 2
    got = [hashlib.sha256(bytes(dst[last, j].cpu().numpy())).digest() for j in (0, k - 1)]
    assert got == [expected[0], expected[k - 1]], 'decoded bytes differ from the source'
    dec_all, stored_all = sum_over_ranks([k * raw * args.steps, len(host) * args.steps], world)
    value = dec_all / (ms / 1e3) / 1e9
    line = {
        'metric': 'decoded MXFP4 expert GB/s into HBM', 'value': round(value, 3), 'unit': 'GB/s', 'n_gpus': world,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(ms / args.steps, 3),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'experts_per_s': round(k * world * args.steps / (ms / 1e3), 1),
        'config': {'workload': f'wnr4: WNR4 kind-MX records (draft codec 8, G = 32, canonical zero) of {k} experts of '
                               f'hidden {cfg["hidden"]}, FFN {cfg["ffn"]} per rank, decoded every step by '
                               f'wnr4_cuda_batch_submit / wait, {B} records per call, up to {depth} calls in flight, '
                               f'from pinned host memory',
                   'l2': 'inputs larger than L2 (126 MB) between steps'},
        'e2e': {'value': round(value, 3), 'unit': 'GB/s', 'h2d_bytes_per_step': int(len(host)), 'd2h_bytes_per_step': 4 * k,
                'roofline': {'bound': 'h2d', 'achieved': round(stored_all / (ms / 1e3) / 1e9 / world, 2),
                             'peak': round(h2d_gbs, 2),
                             'frac': round(stored_all / (ms / 1e3) / 1e9 / world / h2d_gbs, 4)}},
        'gpu_launches': len(calls[0]) * args.steps,
        'clocks': clk, 'verified_records': 2,
    }
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


# ---- expert misses from a container file (config "file") ------------------------------------------------
def file_dir():
    return os.environ.get('WEXB_FILE_DIR') or None


def write_expert_file(cfg, rank, world, threads):
    """This rank's container file: every expert of its shard (expert id mod world size) of cfg['layers']
    layers as WNR3 records under one WNM2 model. Returns (path, owners, experts, model blob)."""
    import tempfile
    import wex4file
    owners = [(l, e) for l in range(cfg['layers']) for e in range(rank, cfg['experts'], world)]
    blob, experts = build_pool(cfg, owners, threads)
    recs = [wex4file.expert_record(e, 0, value_exact=cfg['cz']) for e in experts]
    data = wex4file.write(recs, [(wex4file.BLOB_WNM2, fnv1a(blob), blob)], grid=(cfg['layers'], cfg['experts']),
                          value_exact=cfg['cz'])
    del recs
    fd, path = tempfile.mkstemp(prefix=f'wexb-experts-r{rank}-', suffix='.wex4', dir=file_dir())
    with os.fdopen(fd, 'wb') as f:
        f.write(data)
        f.flush()
        os.fsync(f.fileno())
    return path, owners, experts, blob


def file_record_offsets(path):
    """{(layer, expert): offset} of the expert records, from the container's record table."""
    import struct
    with open(path, 'rb') as fh:
        head = fh.read(4096)
        index_offset, = struct.unpack_from('<Q', head, 32)
        nblobs, nrecords = struct.unpack_from('<II', head, 48)
        fh.seek(index_offset + 64 * nblobs)
        rows = fh.read(72 * nrecords)
    out = {}
    for r in range(nrecords):
        offset, stored, decoded, codec, flags, blob, owner = struct.unpack_from('<QIIHHII', rows, 72 * r)
        if flags & 2:
            out[(owner >> 16, owner & 0xffff)] = offset
    return out


def miss_keys(owners, misses, step):
    """The experts one step reads: `misses` distinct records of the file in a seeded random order."""
    perm = np.random.default_rng(SEED + 7919 * step).permutation(len(owners))[:misses]
    return [owners[int(i)] for i in perm]


def open_expert_file(wexcuda, path):
    """(file, direct): O_DIRECT when the filesystem allows it, else through the page cache."""
    try:
        return wexcuda.ExpertFile(path, direct=True), True
    except OSError as e:
        if e.errno != 1:
            raise
        return wexcuda.ExpertFile(path, direct=False), False


def run_file(args, cfg):
    import torch
    world, rank, local = dist_init()
    torch.cuda.set_device(local)
    threads = max(1, (os.cpu_count() or 8) // max(1, int(os.environ.get('LOCAL_WORLD_SIZE', world))))
    t0 = time.time()
    path, owners, experts, _ = write_expert_file(cfg, rank, world, threads)
    log(f'[rank {rank}] file of {len(owners)} records ({os.path.getsize(path) / 1e9:.2f} GB) written in '
        f'{time.time() - t0:.1f} s at {path}')
    try:   # the file is removed however the run ends
        return file_steps(args, cfg, world, rank, local, path, owners, experts)
    finally:
        if os.path.exists(path):
            os.remove(path)


def file_steps(args, cfg, world, rank, local, path, owners, experts):
    import torch
    import wexcuda
    by_owner = {(e.layer, e.index): e for e in experts}
    raw = len(experts[0].expected)
    N = min(cfg['misses'], len(owners))
    steps = [miss_keys(owners, N, s) for s in range(args.warmup + args.steps)]
    last = steps[-1]
    expected = {k: hashlib.sha256(by_owner[k].expected).digest() for k in (last[0], last[-1])}
    stored = [sum(len(by_owner[k].record) for k in keys) for keys in steps]
    del experts, by_owner
    f, direct = open_expert_file(wexcuda, path)
    dst = torch.empty((N, raw), dtype=torch.uint8, device='cuda')
    import synth
    entry = synth.expert_entry(cfg['hidden'], cfg['ffn'])
    soff = [int.from_bytes(entry[44 + 4 * m:48 + 4 * m], 'little') for m in range(3)]
    woff = [int.from_bytes(entry[56 + 4 * m:60 + 4 * m], 'little') for m in range(3)]
    ds = [dst.data_ptr() + j * raw + soff[m] for j in range(N) for m in range(3)]
    dw = [dst.data_ptr() + j * raw + woff[m] for j in range(N) for m in range(3)]

    def timed(fn, keys):
        if not direct:
            f.evict()
        barrier(world)
        torch.cuda.synchronize()
        t = time.perf_counter()
        fn(keys)
        torch.cuda.synchronize()
        return max_over_ranks(time.perf_counter() - t, world)

    def decode(keys):
        bad, st = f.decode(keys, local, ds, dw)
        assert bad == 0, st

    def read(keys):
        bad, st, got = f.read(keys)
        assert bad == 0, st
    for s in range(args.warmup):
        timed(read, steps[s])
        timed(decode, steps[s])
    h2d_gbs = measure_h2d(torch)
    clocks = Clocks(local)
    clocks.start()
    t_dec = [timed(decode, steps[args.warmup + s]) for s in range(args.steps)]
    clk = clocks.stop()
    t_read = [timed(read, steps[args.warmup + s]) for s in range(args.steps)]
    got = {k: hashlib.sha256(bytes(dst[j].cpu().numpy())).digest() for j, k in ((0, last[0]), (N - 1, last[-1]))}
    assert got == expected, 'decoded bytes differ from the source'
    dec_all, stored_all = sum_over_ranks([N * raw * args.steps, sum(stored[args.warmup:])], world)
    sec, rsec = sum(t_dec), sum(t_read)
    value = dec_all / sec / 1e9
    read_gbs = stored_all / rsec / 1e9 / world
    achieved = stored_all / sec / 1e9 / world
    line = {
        'metric': 'decoded MXFP4 expert GB/s into HBM', 'value': round(value, 3), 'unit': 'GB/s', 'n_gpus': world,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(1e3 * sec / args.steps, 3),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'experts_per_s': round(N * world * args.steps / sec, 1),
        'config': {'workload': f'file: expert misses from a WEX4 container file, {N} distinct WNR3 MXFP4 experts per '
                               f'step in a seeded random order (hidden {cfg["hidden"]}, FFN {cfg["ffn"]}), of a file of '
                               f'{len(owners)} experts per rank ({cfg["layers"]} layers, expert id mod world size), '
                               f'read, uploaded and decoded by wexb_file_decode',
                   'reads': 'O_DIRECT' if direct else 'page cache, evicted before every step',
                   'readers': 8, 'placement': 'expert id mod world size',
                   'l2': 'inputs larger than L2 (126 MB) between steps'},
        'e2e': {'value': round(value, 3), 'unit': 'GB/s', 'h2d_bytes_per_step': int(sum(stored[args.warmup:]) / args.steps),
                'd2h_bytes_per_step': 4 * N, 'api': 'wexb_file_decode (file to HBM)'},
        'roofline': {'bound': 'storage read', 'achieved': round(achieved, 3), 'peak': round(read_gbs, 3),
                     'unit': 'GB/s (stored bytes per GPU)', 'frac': round(achieved / read_gbs, 4),
                     'peak_source': 'measured here: the same records through wexb_file_read (reads alone, same '
                                    'readers and ring), the slowest rank', 'h2d_gbs': round(h2d_gbs, 2)},
        'gpu_launches': 3 * -(-N // 8), 'clocks': clk, 'verified_records': 2,
    }
    f.close()
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            line['cpu_baseline'] = reference_file_miss_rate(args, cfg, None, seconds=args.cpu_seconds)
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def reference_file_miss_rate(args, cfg, built, seconds):
    """The reference's miss path on the host cores: each thread preads one whole record (O_DIRECT when the
    filesystem allows it, as c/expert_store_wex.c opens its file) and decodes it with the reference's CPU
    decoder (oracle/_ref/wex_nr3_tools.so), until `seconds` of work. built: write_expert_file's result, or
    None to write a file of the config's first layer."""
    sys.path.insert(0, os.path.join(ROOT, 'oracle'))
    import ctypes
    import mmap
    import oracle
    L = oracle.ref_lib('wex_nr3_tools')
    if L is None:
        raise RuntimeError('oracle/_ref/wex_nr3_tools.so is missing: build it with `make -C oracle ref`')
    cores = os.cpu_count() or 1
    own = built is None
    if own:
        built = write_expert_file(dict(cfg, layers=1), 0, 1, cores)
    path, owners, experts, blob = built
    by_owner = {(e.layer, e.index): e for e in experts}
    offsets = file_record_offsets(path)
    try:
        fd, direct = os.open(path, os.O_RDONLY | os.O_DIRECT), True
    except OSError:
        fd, direct = os.open(path, os.O_RDONLY), False
    largest = max(len(e.record) for e in experts)
    bufs = [mmap.mmap(-1, largest) for _ in range(cores)]   # page-aligned, as O_DIRECT needs
    outs = [ctypes.create_string_buffer(experts[0].raw) for _ in range(cores)]

    def one(i, key):
        e, b = by_owner[key], bufs[i % cores]
        if os.preadv(fd, [b], offsets[key]) < len(e.record):
            raise RuntimeError('short read')
        rec = (ctypes.c_char * len(e.record)).from_buffer(b)
        st = L.wex_nr3_decode(blob, e.entry, rec, e.layer, e.index, outs[i % cores])
        del rec
        if st != 0:
            raise RuntimeError('reference decoder refused a record')
        return e.raw
    t0, n, nbytes, s = time.perf_counter(), 0, 0, 0
    with ThreadPoolExecutor(cores) as pool:
        while time.perf_counter() - t0 < seconds:
            keys = miss_keys(owners, cores, s)
            s += 1
            nbytes += sum(pool.map(one, range(len(keys)), keys))
            n += len(keys)
    dt = time.perf_counter() - t0
    os.close(fd)
    if own:
        os.remove(path)
    return {'value': round(nbytes / dt / 1e9, 4), 'unit': 'GB/s', 'cores': cores, 'kind': 'reference',
            'sample': f'{n} expert misses ({nbytes / 1e9:.2f} GB decoded) in {dt:.1f} s: one pread of the whole '
                      f'record ({"O_DIRECT" if direct else "page cache"}) then the reference wex_nr2_decode, one '
                      f'record per host thread'}


def run_reference_file(args, cfg):
    """The reference arm of the file config: rank 0 writes the same file and serves each step's misses with
    the reference's path (pread, then its CPU decoder), on all host cores; each step a bounded sample."""
    cores = os.cpu_count() or 1
    built = write_expert_file(cfg, 0, 1, cores)
    N = min(cfg['misses'], len(built[1]))
    raw = built[2][0].raw
    rate = reference_file_miss_rate(args, cfg, built, seconds=args.cpu_seconds)
    os.remove(built[0])
    value = rate['value']
    line = {
        'impl': 'reference', 'metric': 'decoded MXFP4 expert GB/s into HBM', 'value': value, 'unit': 'GB/s',
        'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(1e3 * N * raw / (value * 1e9), 3),
        'experts_per_s': round(value * 1e9 / raw, 2), 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'config': {'workload': f'file: expert misses from a WEX4 container file, {N} distinct WNR3 MXFP4 experts per '
                               f'step (hidden {cfg["hidden"]}, FFN {cfg["ffn"]})'},
        'cpu_baseline': rate,
        'e2e': {'value': value, 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line))
    return 0


# ---- the writer side (config "encode") ---------------------------------------------------------------
def encode_pool(cfg, threads):
    """The coded experts of the encode config (layers x experts, one sigma per layer) and the model
    trained on all of them by the writer tools."""
    import synth
    sig = layer_sigmas(cfg)
    owners = [(l, e) for l in range(cfg['layers']) for e in range(cfg['experts'])]
    with ThreadPoolExecutor(threads) as pool:
        ex = list(pool.map(lambda o: synth.Expert(cfg['hidden'], cfg['ffn'], o[0], o[1], SEED * 17 + o[0] * 4099 + o[1],
                                                  sig[o[0]], cfg['cz'], 0, cfg['neg_zero']), owners))
    blob = synth.train_model([(e.entry, e.coded) for e in ex])
    return ex, blob


def run_encode(args, cfg):
    """Each step counts the training symbols of the step's experts (wexb_count_batch) and encodes them as
    WNR3 records (wexb_encode_batch, chunks 2048:512), from host memory and back: the writer's work for
    one container of `batch` experts."""
    import torch
    import synth
    import wexcuda
    world, rank, local = dist_init()
    torch.cuda.set_device(local)
    threads = max(1, (os.cpu_count() or 8) // max(1, int(os.environ.get('LOCAL_WORLD_SIZE', world))))
    t0 = time.time()
    ex, blob = encode_pool(cfg, threads)
    log(f'[rank {rank}] {len(ex)} coded experts in {time.time() - t0:.1f} s')
    # inputs and outputs in page-locked host memory, as a writer would stage them
    size = len(ex[0].coded)
    host_in = np.empty(len(ex) * size, np.uint8)
    host_out = np.empty(len(ex) * size, np.uint8)   # a record is smaller than its slab or stored RAW
    for i, e in enumerate(ex):
        host_in[i * size:(i + 1) * size] = np.frombuffer(e.coded, np.uint8)
    assert wexcuda.host_register(host_in) == 0 and wexcuda.host_register(host_out) == 0
    coded = [host_in[i * size:(i + 1) * size] for i in range(len(ex))]
    outs = [host_out[i * size:(i + 1) * size] for i in range(len(ex))]
    entries, flags, owners = [e.entry for e in ex], [e.flags for e in ex], [e.owner for e in ex]
    src = len(host_in)
    check = [synth.encode(blob, ex[i].entry, ex[i].coded, ex[i].flags, ex[i].owner)[1] for i in (0, len(ex) - 1)]

    def step():
        st, wc, sc = wexcuda.count_batch(entries, coded, True, local)
        assert st == [0] * len(ex)
        res = wexcuda.encode_batch(blob, entries, coded, flags, owners, True, 2048, 512, local, outs=outs)
        assert all(r[0] in (0, 1) for r in res)
        return res
    for _ in range(args.warmup):
        step()
    clocks = Clocks(local)
    clocks.start()
    times = []
    for _ in range(args.steps):
        barrier(world)
        torch.cuda.synchronize()
        t = time.perf_counter()
        res = step()
        torch.cuda.synchronize()
        times.append(max_over_ranks(time.perf_counter() - t, world))
    clk = clocks.stop()
    got = [outs[i][:res[i][3]].tobytes() for i in (0, len(ex) - 1)]
    assert got == check, 'GPU records differ from the CPU encoder'
    out_bytes = sum(r[3] for r in res if r[0] == 0)
    sec = sum(times)
    value = src * world * args.steps / sec / 1e9
    line = {
        'metric': 'coded MXFP4 expert GB/s counted and encoded into WNR3 records', 'value': round(value, 3),
        'unit': 'GB/s', 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': round(1e3 * sec / args.steps, 3), 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'config': {'workload': f'encode: {len(ex)} coded MXFP4 experts per rank (hidden {cfg["hidden"]}, FFN '
                               f'{cfg["ffn"]}, canonical zero), training counts then WNR3 records (chunks 2048:512) '
                               f'under one WNM2 model, from host memory and back',
                   'l2': 'inputs larger than L2 (126 MB) between steps'},
        'e2e': {'value': round(value, 3), 'unit': 'GB/s', 'h2d_bytes_per_step': 2 * src, 'd2h_bytes_per_step': out_bytes,
                'api': 'wexb_count_batch + wexb_encode_batch'},
        'gpu_launches': 2 + 4, 'clocks': clk, 'verified_records': 2,
    }
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            line['cpu_baseline'] = reference_encode_rate(ex, blob, args.cpu_seconds)
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def reference_encode_rate(ex, blob, seconds):
    """The reference's writer on the host cores: its counts (wex_nr3_count_expert) and its encoder
    (wex_nr3_encode_record) from oracle/_ref/wex_nr3_tools.so, one expert per thread, until `seconds`."""
    sys.path.insert(0, os.path.join(ROOT, 'oracle'))
    import ctypes
    import oracle
    L = oracle.ref_lib('wex_nr3_tools')
    if L is None:
        raise RuntimeError('oracle/_ref/wex_nr3_tools.so is missing: build it with `make -C oracle ref`')
    cores = os.cpu_count() or 1
    cap = 4 * len(ex[0].coded) + 65536
    outs = [ctypes.create_string_buffer(cap) for _ in range(cores)]

    def one(i):
        e = ex[i % len(ex)]
        wc = np.zeros(3 * 567 * 16, np.uint64)
        sc = np.zeros(3 * 256, np.uint64)
        if L.wex_nr3_count_expert(e.entry, e.coded, wc.ctypes.data, sc.ctypes.data) != 0:
            raise RuntimeError('reference counts refused an expert')
        used, total = ctypes.c_size_t(), ctypes.c_size_t()
        if L.wex_nr3_encode_record(blob, e.entry, e.coded, e.flags, e.owner, 2048, 512, outs[i % cores], cap,
                                   ctypes.byref(used), ctypes.byref(total)) < 0:
            raise RuntimeError('reference encoder refused an expert')
        return len(e.coded)
    t0, n, nbytes = time.perf_counter(), 0, 0
    with ThreadPoolExecutor(cores) as pool:
        while time.perf_counter() - t0 < seconds:
            nbytes += sum(pool.map(one, range(n, n + cores)))
            n += cores
    dt = time.perf_counter() - t0
    return {'value': round(nbytes / dt / 1e9, 4), 'unit': 'GB/s', 'cores': cores, 'kind': 'reference',
            'sample': f'{n} experts counted and encoded in {dt:.1f} s, one expert per host thread (reference '
                      f'wex_nr3_count_expert + wex_nr3_encode_record)'}


def run_reference_encode(args, cfg):
    ex, blob = encode_pool(cfg, os.cpu_count() or 1)
    rate = reference_encode_rate(ex, blob, args.cpu_seconds)
    value = rate['value']
    src = len(ex[0].coded)
    line = {
        'impl': 'reference', 'metric': 'coded MXFP4 expert GB/s counted and encoded into WNR3 records', 'value': value,
        'unit': 'GB/s', 'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': round(1e3 * src * len(ex) / (value * 1e9), 3), 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'config': {'workload': f'encode: {len(ex)} coded MXFP4 experts (hidden {cfg["hidden"]}, FFN {cfg["ffn"]}, '
                               f'canonical zero), training counts then WNR3 records (chunks 2048:512)'},
        'cpu_baseline': rate,
        'e2e': {'value': value, 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line))
    return 0


# ---- WEX4 containers (tiny-file, mixed) --------------------------------------------------------------
def container_owners(cfg, rank, world, layers):
    """The experts of this rank's container: tiny-file all of them, mixed one routed step of its shard."""
    if cfg['experts'] <= 16:
        return [(0, i) for i in range(cfg['experts'])]
    trace = routing_trace(cfg, 1, rank, world, layers)
    return sorted({(l, int(e)) for l in range(layers) for e in trace[0][l]})


def codec_plan(cfg, owners):
    """Per owner: 0 RAW (uniform-random nibbles), 8 WNR4, 5 WNR3, by a seeded draw."""
    if 'raw' in cfg:
        return [0 if i in cfg['raw'] else 5 for i in range(len(owners))]
    rng = np.random.default_rng([SEED, 77])
    u = rng.random(len(owners))
    return [0 if x < cfg['raw_frac'] else 8 if x < cfg['raw_frac'] + cfg['wnr4_frac'] else 5 for x in u]


def build_container(cfg, owners, threads, verify_n=12):
    """(file bytes, decoded bytes, codec counts, verification file, its expected digest). The
    verification file holds the first verify_n records (every codec) with their expected digest."""
    import synth
    import wex4file
    sig = layer_sigmas(cfg)
    plan = codec_plan(cfg, owners)
    seed = lambda l, i: SEED * 1000003 + l * 4099 + i
    mk = lambda k: synth.Expert(cfg['hidden'], cfg['ffn'], owners[k][0], owners[k][1], seed(*owners[k]), sig[owners[k][0]],
                                cfg['cz'], 1 if plan[k] == 0 else 0, cfg['neg_zero'])
    layers = sorted({l for l, _ in owners})
    train = [synth.Expert(cfg['hidden'], cfg['ffn'], l, 100000 + l, seed(l, 100000), sig[l], cfg['cz'], 0, cfg['neg_zero'])
             for l in layers[:8]]
    blob = synth.train_model([(e.entry, e.coded) for e in train])
    blob4 = synth.train_model4([(e.entry, e.coded) for e in train[:4]]) if 8 in plan else None
    del train

    def make(k):
        e = mk(k)
        if plan[k] == 8:
            rec = synth.encode4(blob4, e.entry, e.coded, e.flags, k, 32)   # owner = the record's index
            r = wex4file.expert_record(e, 1, codec=wex4file.CODEC_WNR4, stored=rec) if rec else None
        else:
            r = None
        if r is None:
            e.encode(blob)
            r = wex4file.expert_record(e, 0, value_exact=cfg['cz'])
        keep = e.expected if k < verify_n else None
        return r, len(e.source), keep
    with ThreadPoolExecutor(threads) as pool:
        made = list(pool.map(make, range(len(owners))))
    recs = [m[0] for m in made]
    blobs = [(wex4file.BLOB_WNM2, fnv1a(blob), blob)] + ([(wex4file.BLOB_WNM4, fnv1a(blob4), blob4)] if blob4 else [])
    grid = (cfg['layers'], cfg['experts'])
    data = wex4file.write(recs, blobs, grid=grid, value_exact=cfg['cz'])
    counts = {c: sum(1 for r in recs if r.codec == c) for c in (0, 5, 8)}
    vrecs = recs[:verify_n]   # a prefix keeps every WNR4 record at its own index (its owner)
    vdata = wex4file.write(vrecs, blobs, grid=grid, value_exact=cfg['cz'])
    vdigest = wex4file.content_digest(vrecs, [m[2] for m in made[:verify_n]])
    return data, sum(m[1] for m in made), counts, vdata, vdigest


def fnv1a(b):
    h = 2166136261
    for x in b:
        h = ((h ^ x) * 16777619) & 0xffffffff
    return h or 1


def run_container(args, cfg):
    import ctypes
    import torch
    import wexcuda
    world, rank, local = dist_init()
    torch.cuda.set_device(local)
    layers = args.layers or cfg['layers']
    threads = max(1, (os.cpu_count() or 8) // max(1, int(os.environ.get('LOCAL_WORLD_SIZE', world))))
    owners = container_owners(cfg, rank, world, layers)
    t0 = time.time()
    data, decoded, counts, vdata, vdigest = build_container(cfg, owners, threads)
    log(f'[rank {rank}] container of {len(owners)} records ({len(data) / 1e9:.2f} GB, codecs {counts}) built in '
        f'{time.time() - t0:.1f} s')
    L = wexcuda.lib()
    L.wex4_check.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_void_p]
    buf = np.frombuffer(data, np.uint8).copy()
    del data
    assert wexcuda.host_register(buf) == 0
    vbuf = np.frombuffer(vdata, np.uint8).copy()
    digest = ctypes.create_string_buffer(32)
    # verification (untimed): the digest of the first records equals the one of their source slabs
    assert L.wex4_check(vbuf.ctypes.data, len(vbuf), 1 | 2 | 4, digest) == 0, 'verification file refused'
    assert digest.raw == vdigest, 'content digest differs'
    flags = 1 | 2 | 4 | 8   # record hashes, decode, codec 8; the digest is the untimed verification above
    barrier(world)
    h2d_gbs = min_over_ranks(measure_h2d(torch), world)   # every rank copying at once
    for _ in range(args.warmup):
        assert L.wex4_check(buf.ctypes.data, len(buf), flags, digest) == 0
    clocks = Clocks(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        assert L.wex4_check(buf.ctypes.data, len(buf), flags, digest) == 0
    torch.cuda.synchronize()
    dt = max_over_ranks(time.perf_counter() - t0, world)
    barrier(world)
    clk = clocks.stop()
    # the two halves of a check, each alone (one call each, after the timed region): hashes only, and
    # decodes only
    parts = {}
    for name, fl in (('hashes_only_ms', 1), ('decode_only_ms', flags & ~1)):
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        assert L.wex4_check(buf.ctypes.data, len(buf), fl, digest) == 0
        torch.cuda.synchronize()
        parts[name] = round(1e3 * (time.perf_counter() - t1), 2)
    dec_all, stored_all, recs_all = sum_over_ranks([decoded * args.steps, len(buf) * args.steps, len(owners) * args.steps],
                                                   world)
    value = dec_all / dt / 1e9
    line = {
        'metric': 'decoded MXFP4 expert GB/s into HBM', 'value': round(value, 3), 'unit': 'GB/s', 'n_gpus': world,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(1e3 * dt / args.steps, 3),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'experts_per_s': round(recs_all / dt, 1),
        'config': {'workload': f'{args.config}: WEX4 container per rank, {len(owners)} expert records (hidden '
                               f'{cfg["hidden"]}, FFN {cfg["ffn"]}), codecs {counts}, checked by wex4_check: '
                               f'record SHA-256 against the index, codec dispatch, decode into HBM (the content '
                               f'digest verified once, untimed, on the first records)',
                   'placement': 'expert id mod world size', 'l2': 'inputs larger than L2 (126 MB) between steps'},
        'e2e': {'value': round(value, 3), 'unit': 'GB/s', 'h2d_bytes_per_step': int(len(buf)), 'd2h_bytes_per_step': 32,
                'api': f'wex4_check(file, flags {flags}) from pinned host memory: the whole path',
                'roofline': {'bound': 'h2d', 'achieved': round(len(buf) * args.steps / dt / 1e9, 2), 'peak': round(h2d_gbs, 2),
                             'frac': round(len(buf) * args.steps / dt / 1e9 / h2d_gbs, 4)}},
        'clocks': clk,
        'verified': {'digest_records': min(12, len(owners)), 'statuses': 'all 0'},
        'parts': parts,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        dt, n, nb = reference_file_rate(bytes(buf), cores, min_seconds=args.cpu_seconds)
        line['cpu_baseline'] = {'value': round(nb / dt / 1e9, 4), 'unit': 'GB/s', 'cores': cores, 'kind': 'reference',
                                'experts_per_s': round(n / dt, 2),
                                'sample': f'{n} records of the same file, one per host thread: the reference tool\'s '
                                          f'wex4_decode_record_buf (SHA-256, then decode; codec 8: SHA-256 and the '
                                          f'reference WNR4 decoder), {dt:.1f} s'}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def measure_h2d(torch, mib=256, reps=5):
    """Pinned host-to-device copy bandwidth of this GPU (GB/s), best of reps, CUDA events."""
    src = torch.empty(mib << 20, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(mib << 20, dtype=torch.uint8, device='cuda')
    best = 0.0
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        best = max(best, (mib << 20) / (a.elapsed_time(b) / 1e3) / 1e9)
    return best


def measure_h2d_calls(torch, views, calls, reps=3):
    """Pinned host-to-device bandwidth (GB/s) of the copies the end-to-end calls issue: each call's records
    copied one cudaMemcpyAsync each, in call order, into a device buffer of one call's records, on one
    stream; best of reps over all calls of a step (CUDA events)."""
    cap = max(sum(len(views[i]) for i in c) for c in calls)
    dst = torch.empty(cap, dtype=torch.uint8, device='cuda')
    srcs = [[torch.from_numpy(views[i]) for i in c] for c in calls]
    total = sum(int(t.numel()) for c in srcs for t in c)
    best = 0.0
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for c in srcs:
            at = 0
            for t in c:
                n = int(t.numel())
                dst[at:at + n].copy_(t, non_blocking=True)
                at += n
        b.record()
        torch.cuda.synchronize()
        best = max(best, total / (a.elapsed_time(b) / 1e3) / 1e9)
    del dst
    return best


def profile_value(config, key):
    """A figure of the decode kernel's committed ncu summary (a `key: value` line), if there is one."""
    path = os.path.join(ROOT, 'profiles', f'nr3_decode_{config}.md')
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith(key + ':'):
            return float(line.split(':')[1])
    return None


def profile_traffic_per_record(config):
    """DRAM bytes per record of the decode kernel from its committed ncu summary, if there is one."""
    v = profile_value(config, 'traffic_bytes_per_record')
    return int(v) if v else None


def config_desc(args, cfg, records):
    if cfg.get('all_experts'):
        return {'workload': f'{args.config}: streaming decode of every expert of the rank\'s shard (expert id mod '
                            f'world size) each step, WNR3 MXFP4 experts, hidden {cfg["hidden"]}, expert FFN {cfg["ffn"]}, '
                            f'{cfg["layers"] * cfg["experts"]} experts in all' + (', canonical zero' if cfg['cz'] else ''),
                'records_per_step_per_gpu': records, 'chunks': '2048:512', 'placement': 'expert id mod world size',
                'l2': 'inputs larger than L2 (126 MB) between steps'}
    return {'workload': f'{args.config}: routed decode of WNR3 MXFP4 experts, hidden {cfg["hidden"]}, expert FFN '
                        f'{cfg["ffn"]}, {args.layers or cfg["layers"]} layers x {cfg["experts"]} experts, top-'
                        f'{cfg["batch"]} Zipf(1.1) per layer per step' + (', canonical zero' if cfg['cz'] else '') +
                        (f', {cfg["trace_steps"]} distinct routing step(s) cycled' if cfg.get('trace_steps') else ''),
            'records_per_step_per_gpu': records,
            'chunks': '2048:512', 'placement': 'expert id mod world size',
            'l2': 'inputs larger than L2 (126 MB) between steps'}


def gpu_reference_rate(args, blob, call_args, steps_total, check):
    """The reference's own CUDA helper (c/tools/wex_cuda_bridge.cu compiled unchanged for sm_100a into
    oracle/_ref/libwex_cuda_ref.so) on the same pinned records, destinations and calls as the
    synchronous drop-in form of e2e: per layer one wex_cuda_decode_batch_to_device of `batch` records.
    A yardstick beside this library on the same GPU, never part of it. Times as many of the timed
    steps as fit about 20 s (host clock, device synchronised), then checks the sampled slabs with
    check(). Returns a dict, or one saying why it did not run."""
    import ctypes
    import torch
    path = os.path.join(ROOT, 'oracle', '_ref', 'libwex_cuda_ref.so')
    if not os.path.exists(path):
        return {'unavailable': 'oracle/_ref/libwex_cuda_ref.so was not built (make -C oracle gpuref)'}
    R = ctypes.CDLL(path)
    P, I = ctypes.c_void_p, ctypes.c_int
    R.wex_cuda_helper_abi.restype = ctypes.c_uint
    R.wex_cuda_register_model.argtypes = [P, ctypes.c_size_t]
    R.wex_cuda_decode_batch_to_device.argtypes = [I, P, P, I, P, P, P]
    if R.wex_cuda_helper_abi() != 1 or R.wex_cuda_register_model(blob, len(blob)) != 0:
        return {'unavailable': 'the reference helper refused its ABI check or the model'}
    dev = torch.cuda.current_device()

    def step(s):
        bad = 0
        for ep, rp, sp, wp, st, _ in call_args[s]:
            bad += R.wex_cuda_decode_batch_to_device(len(st), ep, rp, dev, sp, wp, st)
        return bad
    for s in range(args.warmup):
        assert step(s) == 0, 'the reference helper refused a record'
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert step(args.warmup) == 0
    torch.cuda.synchronize()
    first = time.perf_counter() - t0
    n = max(1, min(args.steps, int(20.0 / max(first, 1e-6))))
    t0 = time.perf_counter()
    for s in range(args.warmup, args.warmup + n):
        assert step(s) == 0
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    ok = check(args.warmup + n - 1)
    return {'steps': n, 'seconds': dt, 'verified': ok}


def run_gpu(args, cfg):
    import torch
    import wexcuda
    world, rank, local = dist_init()
    torch.cuda.set_device(local)
    dev = local
    numa = bind_to_gpu_numa_node(local) if world > 1 else None
    layers = args.layers or cfg['layers']
    steps_total = args.warmup + args.steps
    trace = routing_trace(cfg, steps_total, rank, world, layers)
    owners = sorted({(l, int(e)) for s in range(steps_total) for l in range(layers) for e in trace[s][l]})
    local_world = max(1, int(os.environ.get('LOCAL_WORLD_SIZE', world)))
    if numa is not None:   # the node's CPUs shared by the ranks bound to it
        nodes = sum(1 for d in os.listdir('/sys/devices/system/node') if d.startswith('node') and d[4:].isdigit())
        threads = max(1, len(os.sched_getaffinity(0)) // max(1, -(-local_world // max(1, nodes))))
    else:
        threads = max(1, (os.cpu_count() or 8) // local_world)
    t0 = time.time()
    blob, experts = build_pool(cfg, owners, threads, device=dev)
    log(f'[rank {rank}] {len(experts)} experts generated and encoded in {time.time() - t0:.1f} s')
    assert all(e.codec == 5 for e in experts), 'every synthetic expert compresses'
    index = {(e.layer, e.index): i for i, e in enumerate(experts)}
    assert wexcuda.register_model(blob) == 0
    hostbuf, views = pinned_records(experts)
    raw = experts[0].raw
    k = sum(len(trace[0][l]) for l in range(layers))   # records per step
    # destinations of one step: 384 experts' six regions
    sizes = [r * c // 32 for r, c in [(cfg['ffn'], cfg['hidden']), (cfg['hidden'], cfg['ffn']), (cfg['ffn'], cfg['hidden'])]]
    dst = torch.empty((k, raw), dtype=torch.uint8, device='cuda')
    base = dst.data_ptr()
    soffs = [0, sizes[0], sizes[0] + sizes[1]]
    woffs = [sum(sizes) + 16 * x for x in soffs]
    dscale = [base + j * raw + soffs[m] for j in range(k) for m in range(3)]
    dweight = [base + j * raw + woffs[m] for j in range(k) for m in range(3)]
    step_idx = [[index[(l, int(e))] for l in range(layers) for e in trace[s][l]] for s in range(steps_total)]

    # ---- value: resident records, one decode per step --------------------------------------------
    res = wexcuda.Resident([e.entry for e in experts], views, dev)
    assert res.failures == 0
    res.profile(True)
    h2d_gbs = measure_h2d(torch)
    barrier(world)
    h2d_together = min_over_ranks(measure_h2d(torch), world) if world > 1 else h2d_gbs   # every rank copying at once
    # the same link with the copies the end-to-end calls make (a call's records, one copy each), every rank at once
    step_calls = [step_idx[0][c:c + cfg['batch']] for c in range(0, k, cfg['batch'])]
    barrier(world)
    h2d_calls = min_over_ranks(measure_h2d_calls(torch, views, step_calls), world)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    kernel_ms, launches = [], 0
    for s in range(args.warmup):
        assert res.decode(step_idx[s], dscale, dweight, sh) == 0
        bad, st = res.wait()
        assert bad == 0, st
    clocks = Clocks(dev)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for s in range(args.warmup, steps_total):   # two decodes queued: step s is planned while s - 1 runs
        assert res.decode(step_idx[s], dscale, dweight, sh) == 0
        launches += res.launches()
        if s > args.warmup:
            bad, st = res.wait()
            assert bad == 0, st
            kernel_ms.append(res.kernel_ms())
    bad, st = res.wait()
    assert bad == 0, st
    kernel_ms.append(res.kernel_ms())
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    value_ms = max_over_ranks(ev0.elapsed_time(ev1), world)
    # bit-exact check of the last step's slabs (8 sampled records)
    last = step_idx[steps_total - 1]
    check = list(range(0, k, max(1, k // 8)))[:8]
    got = dst[check].cpu().numpy()
    verified = sum(int(hashlib.sha256(got[i].tobytes()).digest() == experts[last[j]].expected_sha)
                   for i, j in enumerate(check))
    assert verified == len(check), 'decoded bytes differ from the source'
    # per-record outcome table of the last step (status, digest of the checked slabs), all ranks
    slab_digest = {j: hashlib.sha256(got[n].tobytes()).hexdigest()[:16] for n, j in enumerate(check)}
    table = gather_outcomes([(rank, experts[i].layer, experts[i].index, int(st[j]), slab_digest.get(j, ''))
                             for j, i in enumerate(last)], world)

    # ---- e2e: 8 records per layer per call, from pinned host memory, statuses read back ------------
    # Argument arrays are built once per (step, layer) as an engine holds them; the timed region
    # covers the calls themselves: uploads, kernels, status read-back.
    import ctypes
    L = wexcuda.lib()
    B = cfg['batch']
    entry_store = [np.frombuffer(bytes(e.entry), np.uint8).copy() for e in experts]
    verify = bool(cfg.get('verify'))
    depth = args.depth or (160 if verify else 3)
    rec_sha = None
    if verify:   # each record's SHA-256, as a WEX4 index keeps it (c/wex4.h:673-677), computed once on the host
        with ThreadPoolExecutor(threads) as pool:
            rec_sha = list(pool.map(lambda e: hashlib.sha256(e.record).digest(), experts))
    # destination sets: calls of two steps in flight at once never share a destination (more calls in
    # flight than a step holds: one set per step that can be in flight, used in turn)
    ncalls = -(-k // B)
    dsts = [dst] + [torch.empty((k, raw), dtype=torch.uint8, device='cuda') for _ in range(depth // ncalls + 1 if depth >= ncalls else 0)]
    def set_ptrs(t):
        b = t.data_ptr()
        return ([b + j * raw + soffs[m] for j in range(k) for m in range(3)], [b + j * raw + woffs[m] for j in range(k) for m in range(3)])
    set_args = [set_ptrs(t) for t in dsts]
    call_args = []
    for s in range(steps_total):
        ids = step_idx[s]
        ds, dw = set_args[s % len(dsts)]
        per = []
        for c in range(0, k, B):   # one call per B records (a layer's batch)
            sel = ids[c:c + B]
            dg = np.frombuffer(b''.join(rec_sha[i] for i in sel), np.uint8).copy() if verify else None
            per.append((wexcuda._ptrs([entry_store[i].ctypes.data for i in sel]),
                        wexcuda._ptrs([views[i].ctypes.data for i in sel]),
                        wexcuda._ptrs(ds[3 * c:3 * (c + B)]), wexcuda._ptrs(dw[3 * c:3 * (c + B)]),
                        (ctypes.c_int * B)(), dg))
        call_args.append(per)
    assert ncalls == len(call_args[0])

    def sync_step(s):
        bad = 0
        for ep, rp, sp, wp, st, _ in call_args[s]:
            bad += L.wex_cuda_decode_batch_to_device(B, ep, rp, dev, sp, wp, st)
        return bad

    def queued_step(s, pending):
        bad = 0
        for ep, rp, sp, wp, st, dg in call_args[s]:
            if verify:   # the record hashes on the GPU before the decode may write the destination
                t = L.wexb_batch_submit_verified(B, ep, rp, dg.ctypes.data, dev, sp, wp)
            else:
                t = L.wexb_batch_submit(B, ep, rp, dev, sp, wp)
            assert t >= 0
            pending.append((t, st))
            if len(pending) > depth:
                t0_, st0 = pending.pop(0)
                bad += L.wexb_batch_wait(t0_, st0)
        return bad

    def drain(pending):
        bad = 0
        while pending:
            t_, st_ = pending.pop(0)
            bad += L.wexb_batch_wait(t_, st_)
        return bad

    def timed(run):
        barrier(world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        run()
        torch.cuda.synchronize()
        dt = max_over_ranks(time.perf_counter() - t0, world)
        barrier(world)
        return dt

    if not verify:
        for s in range(args.warmup):
            assert sync_step(s) == 0
    pend = []
    for s in range(args.warmup):
        assert queued_step(s, pend) == 0
    assert drain(pend) == 0

    def run_queued():
        p, bad = [], 0
        for s in range(args.warmup, steps_total):
            bad += queued_step(s, p)
        bad += drain(p)
        assert bad == 0

    def run_sync():
        assert sum(sync_step(s) for s in range(args.warmup, steps_total)) == 0

    # each end-to-end form is timed three times over the same K steps (the host link is shared with
    # other work on the machine); the median is reported, with every sample
    e2e_runs = [timed(run_queued) for _ in range(3)]
    # a verified call waits for its records' SHA-256 chains: one at a time is a latency figure only
    sync_runs = [timed(run_sync) for _ in range(3)] if not verify else None
    e2e_s = statistics.median(e2e_runs)
    sync_s = statistics.median(sync_runs) if sync_runs else None
    clk = clocks.stop()
    got = dsts[(steps_total - 1) % len(dsts)][check].cpu().numpy()
    assert all(hashlib.sha256(got[i].tobytes()).digest() == experts[last[j]].expected_sha for i, j in enumerate(check))

    # ---- bytes ----------------------------------------------------------------------------------
    dec_bytes = sum(experts[i].raw for s in range(args.warmup, steps_total) for i in step_idx[s])
    stored = sum(len(experts[i].record) for s in range(args.warmup, steps_total) for i in step_idx[s])
    wbytes = sum(int.from_bytes(experts[i].entry[16:20], 'little') + int.from_bytes(experts[i].entry[12:16], 'little')
                 for s in range(args.warmup, steps_total) for i in step_idx[s])
    totals = sum_over_ranks([dec_bytes, stored, k * args.steps], world)
    dec_all, stored_all, recs_all = totals
    value = dec_all / (value_ms / 1e3) / 1e9
    e2e = dec_all / e2e_s / 1e9
    e2e_sync = dec_all / sync_s / 1e9 if sync_s else None
    # roofline of the decode launch (the only kernel of a step: scale, weight and commit items), from
    # algorithmic bytes per launch = records read (stored bytes) + decode-layout slabs written + the
    # error-gated commit (slabs read, destinations written), over its event-timed duration
    dk = [m[1] for m in kernel_ms if m]
    dk_ms = statistics.mean(dk) if dk else None
    alg = (stored + 3 * dec_bytes) / args.steps
    peaks = json.load(open(MEASURED_PEAKS)) if os.path.exists(MEASURED_PEAKS) else {}
    hbm_peak = peaks.get('hbm_gbs', 6650.0)
    achieved = alg / (dk_ms / 1e3) / 1e9 if dk_ms else None
    traffic_rec = profile_traffic_per_record(args.config)
    # the kernel's compute roofline: warp-instructions issued (the ncu count per warp and symbol of the
    # committed profile x the launch's symbols / 32) over the event-timed duration, against the issue rate
    # of every scheduler (4 per SM, one warp-instruction a cycle) at the sampled SM clock
    ipws = profile_value(args.config, 'warp_instructions_per_warp_symbol')
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    issue = None
    symbols = 2 * sum(int.from_bytes(experts[i].entry[16:20], 'little') for s in range(args.warmup, steps_total)
                      for i in step_idx[s])   # two weight symbols per packed byte
    if ipws and dk_ms and clk.get('sm_mhz'):
        winstr = symbols / args.steps / 32 * ipws
        peak_issue = sms * 4 * clk['sm_mhz'] * 1e6
        issue = {'bound': 'warp-instruction issue', 'achieved': round(winstr / (dk_ms / 1e3) / 1e12, 4),
                 'peak': round(peak_issue / 1e12, 4), 'unit': 'T warp-instructions/s',
                 'frac': round(winstr / (dk_ms / 1e3) / peak_issue, 4),
                 'source': f'{ipws} warp-instructions per weight warp-symbol (ncu, committed profile, every item of '
                           f'the launch counted) x weight symbols / 32; {sms} SMs x 4 schedulers at the median '
                           f'sampled SM clock'}
    h2d_per_step = stored // args.steps + 0
    # rooflines of the two paths (per GPU): the resident decode against HBM (records read, slabs written
    # by the decoder and again by the commit copy), the end-to-end path against the measured H2D link
    hbm_bytes = (stored + dec_bytes + 2 * dec_bytes) / args.steps
    step_s = value_ms / 1e3 / args.steps
    e2e_step_s = e2e_s / args.steps
    line = {
        'metric': 'decoded MXFP4 expert GB/s into HBM', 'value': round(value, 3), 'unit': 'GB/s', 'n_gpus': world,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(value_ms / args.steps, 3),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'u8', 'data': 'synthetic',
        'experts_per_s': round(recs_all / (value_ms / 1e3), 1),
        'config': config_desc(args, cfg, k),
        'e2e': {'value': round(e2e, 3), 'unit': 'GB/s', 'experts_per_s': round(recs_all / e2e_s, 1),
                'h2d_bytes_per_step': int(h2d_per_step), 'd2h_bytes_per_step': 4 * k,
                'api': (f'wexb_batch_submit_verified/wexb_batch_wait (every record SHA-256 checked on the GPU '
                        f'against its digest before its decode may write)' if verify else
                        'wexb_batch_submit/wexb_batch_wait') +
                       f', {B} records per call, {ncalls} calls per step, {depth} calls in flight',
                'ms_per_step': round(1e3 * e2e_s / args.steps, 3),
                'gpu_launches': (2 if verify else 1) * ncalls * args.steps,
                'samples_ms_per_step': [round(1e3 * t / args.steps, 3) for t in e2e_runs], 'reported': 'median of 3',
                'sync': ({'value': round(e2e_sync, 3), 'unit': 'GB/s',
                          'api': 'wex_cuda_decode_batch_to_device (drop-in, synchronous)',
                          'ms_per_step': round(1e3 * sync_s / args.steps, 3),
                          'samples_ms_per_step': [round(1e3 * t / args.steps, 3) for t in sync_runs]}
                         if sync_s else {'skipped': 'verified config: one call at a time waits for whole SHA-256 '
                                                    'chains, a latency figure, not this workload'}),
                'roofline': {'bound': 'h2d', 'achieved': round(h2d_per_step / e2e_step_s / 1e9, 2),
                             'peak': round(h2d_calls, 2), 'unit': 'GB/s (stored bytes per GPU)',
                             'frac': round(h2d_per_step / e2e_step_s / 1e9 / h2d_calls, 4),
                             'peak_source': 'measured here: the copies of one step\'s calls (each record one '
                                            'pinned cudaMemcpyAsync, in call order), best of 3, every rank copying '
                                            'at once (the slowest rank)',
                             'peak_one_copy': round(h2d_together, 2),
                             'frac_of_one_copy': round(h2d_per_step / e2e_step_s / 1e9 / h2d_together, 4),
                             'peak_one_gpu': round(h2d_gbs, 2),
                             'hbm_frac': round(hbm_bytes / e2e_step_s / 1e9 / hbm_peak, 4)}},
        # the end-to-end path per GPU, for comparing runs at different N: each GPU's share of the host link
        # (every rank copying at once) bounds it, not a collective
        'e2e_scaling': {'gpus': world, 'decoded_gbs_per_gpu': round(e2e / world, 3),
                        'stored_gbs_per_gpu': round(h2d_per_step / e2e_step_s / 1e9, 2),
                        'h2d_gbs_per_gpu_all_copying': round(h2d_calls, 2),
                        'frac_of_h2d_all_copying': round(h2d_per_step / e2e_step_s / 1e9 / h2d_calls, 4)},
        'value_roofline': {'bound': 'hbm', 'achieved': round(hbm_bytes / step_s / 1e9, 2), 'peak': hbm_peak, 'unit': 'GB/s',
                           'frac': round(hbm_bytes / step_s / 1e9 / hbm_peak, 4),
                           'bytes': 'records read + slabs written by the decoder and by the commit copy'},
        'roofline': {'bound': 'hbm', 'kernel': 'nr3_decode', 'achieved': round(achieved, 2) if achieved else None,
                     'peak': hbm_peak, 'unit': 'GB/s', 'frac': round(achieved / hbm_peak, 5) if achieved else None,
                     'peak_source': 'measured' if peaks else 'fallback',
                     'traffic': int(traffic_rec * k) if traffic_rec else None,
                     'traffic_source': 'ncu dram__bytes_read.sum + dram__bytes_write.sum per record of a smaller '
                                       'launch, scaled to this launch' if traffic_rec else None,
                     'kernel_ms': round(dk_ms, 4) if dk_ms else None,
                     'alg_bytes_per_launch': int(alg),
                     'alg_bytes': 'records read + decode-layout slabs written + commit (slabs read, destinations '
                                  'written): stored + 3 x decoded bytes',
                     'step_ms': dict(zip(('metadata_upload', 'decode', 'status_readback'),
                                         [round(statistics.mean(m[i] for m in kernel_ms if m), 4) for i in range(3)])),
                     'issue': issue},
        'gpu_launches': launches,
        'clocks': clk,
        'verified_records': verified,
        'outcomes': {'records': len(table), 'failed': sum(1 for r in table if r[3]),
                     'verified_slabs': sum(1 for r in table if r[4])},
        'stored_over_decoded': round(stored / dec_bytes, 4),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        dt, n, nb = reference_decode_rate(experts, blob, cores, min_seconds=args.cpu_seconds)
        line['cpu_baseline'] = {'value': round(nb / dt / 1e9, 4), 'unit': 'GB/s', 'cores': cores, 'kind': 'reference',
                                'experts_per_s': round(n / dt, 2),
                                'sample': f'{n} records of the same pool, one per host thread, reference '
                                          f'wex_nr2_decode, {dt:.1f} s'}
        # the stronger comparator: the reference's fast CPU decoder, through its WEX4 tool, on a file of
        # 32 records of the pool
        import wex4file
        sample = sorted({(e.layer, e.index): e for e in experts if e.codec == 5}.values(), key=lambda e: (e.layer, e.index))[:32]
        fdata = wex4file.write([wex4file.expert_record(e, 0, value_exact=cfg["cz"]) for e in sample], [(wex4file.BLOB_WNM2, fnv1a(blob), blob)],
                               grid=(cfg['layers'], cfg['experts']), value_exact=cfg['cz'])
        fdt, fn, fnb = reference_file_rate(fdata, cores, min_seconds=args.cpu_seconds / 2, lib='wex4_tools_fast')
        line['cpu_baseline']['fast'] = {'value': round(fnb / fdt / 1e9, 4), 'unit': 'GB/s', 'cores': cores,
                                        'experts_per_s': round(fn / fdt, 2),
                                        'sample': f'{fn} records, one per host thread: the reference fast decoder '
                                                  f'(wex4_tools built with WEX4_FAST_NR3, SHA-256 checked), {fdt:.1f} s'}
    if rank == 0 and world == 1 and not args.no_gpu_reference:
        def check_step(s):   # the sampled slabs of step s against the source digests
            got_ = dst[check].cpu().numpy()
            ids = step_idx[s]
            return all(hashlib.sha256(got_[n].tobytes()).digest() == experts[ids[j]].expected_sha
                       for n, j in enumerate(check))
        dst.fill_(0xA5)
        g = gpu_reference_rate(args, blob, call_args, steps_total, check_step)
        if 'steps' in g:
            gb = sum(experts[i].raw for s in range(args.warmup, args.warmup + g['steps']) for i in step_idx[s])
            line['gpu_reference'] = {
                'value': round(gb / g['seconds'] / 1e9, 3), 'unit': 'GB/s',
                'experts_per_s': round(k * g['steps'] / g['seconds'], 1),
                'ms_per_step': round(1e3 * g['seconds'] / g['steps'], 3), 'steps': g['steps'],
                'verified_slabs': g['verified'],
                'api': f'the reference CUDA helper (c/tools/wex_cuda_bridge.cu, compiled unchanged for sm_100a): '
                       f'wex_cuda_decode_batch_to_device, {B} records per call, {ncalls} calls per step, from the '
                       f'same pinned records into the same destinations',
                'vs': {'e2e_sync': round(e2e_sync / (gb / g['seconds'] / 1e9), 3) if e2e_sync else None,
                       'e2e': round(e2e / (gb / g['seconds'] / 1e9), 3)}}
            assert g['verified'], 'the reference helper decoded different bytes'
        else:
            line['gpu_reference'] = g
    res.close()
    import resource
    log(f'[rank {rank}] peak host memory {resource.getrusage(resource.RUSAGE_SELF).ru_maxrss / 1e6:.1f} GB')
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=5)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', choices=['wexb', 'reference'], default='wexb')
    ap.add_argument('--config', choices=sorted(CONFIGS), default='large')
    ap.add_argument('--layers', type=int, default=0, help='layers per step (default: all of the config)')
    ap.add_argument('--cpu-seconds', type=float, default=12.0)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-gpu-reference', action='store_true',
                    help='skip the reference CUDA helper timed beside this library (1 GPU)')
    ap.add_argument('--depth', type=int, default=0,
                    help='e2e: batch calls kept in flight (default 3; 160 for a verified config)')
    args = ap.parse_args()
    assert args.warmup >= 1
    cfg = CONFIGS[args.config]
    if args.impl == 'reference':
        return run_reference(args, cfg)
    if cfg.get('container'):
        return run_container(args, cfg)
    if cfg.get('wnr4'):
        return run_wnr4(args, cfg)
    if cfg.get('file'):
        return run_file(args, cfg)
    if cfg.get('encode'):
        return run_encode(args, cfg)
    return run_gpu(args, cfg)


if __name__ == '__main__':
    sys.exit(main())
