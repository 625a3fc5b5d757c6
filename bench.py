"""Benchmark: BirdNET-v2.4-architecture int8 windows/s on B200 (one process per GPU, weak scaling).

    python bench.py [--gpus N --steps K --warmup W --batch B] [--impl reference]
    (N > 1: python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N)

A step scores one batch of B (default 256) windows of 144000 samples through the full v2.4-architecture neon-int8
package (66 ops: front end, c0, p0, 16 blocks, post conv, 6522-class int8 head) on every GPU. The package is written
by bnneon_b200.synth (byte-identical to the reference compiler's output for the same synthetic IR: random
He-normal weights, seeded noise-plus-chirp audio; no network, no real model).

Printed (rank 0, one JSON line):
  value   windows/s of the whole job, inputs resident in HBM (bnn_infer_device), device time (CUDA events on the
          launching stream), max over ranks;
  e2e     the same through bnn_infer_batch with pinned host buffers: host->device PCM and device->host logits and
          embeddings inside the timed region;
  roofline  the op class with the most device time (per-op CUDA events): algorithmic bytes / its time vs the
          measured HBM copy bandwidth (MEASURED_PEAKS.json);
  cpu_baseline  the reference's own C runtime (oracle/_ref: its unmodified sources compiled for x86, NEON intrinsics
          through a scalar stand-in) on this host's cores, a bounded sample of the same windows; the C restatement
          of the reference's path (oracle/liboracle.so) where that build is absent;
  parity_checked  the timed calls' outputs against the CPU oracle, after timing.
`--impl reference` times that CPU implementation alone on rank 0 (the reference arm).
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "birdnet-neon-engine_b200"))
sys.path.insert(0, REPO)

METRIC = "BirdNET-v2.4-arch int8 windows/s at 1/2/4/8 B200; s8 GEMM TOPS vs int8 peak"
UNIT = "windows/s"
WORKLOAD = "BirdNET-v2.4-architecture neon-int8 package (config 2): 144000-sample windows, batch per GPU"

# per-window algorithmic bytes and MACs of each op (read inputs once, write outputs once, weights once per batch)
OPCODE_NAMES = {1: "fe_stft2", 2: "c0pool_f32", 4: "dw3_f32", 6: "postpc_f32", 22: "pw_s8n", 23: "gemv_s8n",
                25: "se_gate_f32"}


def op_cost(code, p, bufs, bl):
    """(bytes per window, weight bytes per batch, int8 MACs per window) of one op record."""
    if code == 22:  # PW_S8: x [M][K] f32 (+ gate), weights, out [M][Np] f32 (+ residual)
        N, K, Kp, Np, M = p[0], p[1], p[2], p[3], p[4]
        by = M * K * 4 + M * Np * 4 + (M * Np * 4 if bl[2] >= 0 else 0) + (K * 4 if len(bl) == 7 and bl[6] >= 0 else 0)
        return by, Np * Kp + Np * 12, M * N * K
    if code == 23:
        N, K, Kp, Np = p[0], p[1], p[2], p[3]
        return K * 4 + Np * 4, Np * Kp + Np * 12, N * K
    if code == 4:  # DW3: haloed input, output, channel sums
        H, W, C, _, Ho, Wo = p[:6]
        return (H * W * C + Ho * Wo * C + C) * 4, 10 * C * 4, 0
    if code == 25:
        C, rd = p[0], p[1]
        return 2 * C * 4, (2 * rd * C + rd + C) * 4, 0
    if code == 2:
        return (96 * 511 * 2 + 6144 * 48) * 4, 25 * 24 * 4, 0
    if code == 6:
        return (24 * 192 + 1024) * 4, 1728 * 1024 * 4, 0
    if code == 1:
        return (144000 + 96 * 511 * 2) * 4, 0, 0
    return 0, 0, 0


PROFILE = os.path.join(REPO, "profiles", "launch_list_v24_int8_b256.md")
NCU_CMD = ("ncu --metrics gpu__time_duration.sum --clock-control none "
           "-s {skip} -c {count} --csv --log-file <out>/launches.csv python bench.py --ncu --warmup 3")
# the kernels each op launches, in order (the runtime's op registry)
OP_KERNELS = {1: ("k_fe_minmax", "k_fe_spec"), 2: ("k_c0pool",), 22: ("k_quant", "k_gemm_s8"),
              23: ("k_quant", "k_gemm_s8"), 4: ("k_dw3",), 25: ("k_se_gate",), 6: ("k_postpc_im2col", "k_postpc_gemm")}


def ncu_summary(csv_path, batch):
    """Reads an ncu launch list (gpu__time_duration.sum, one step of the full package; DRAM byte counters too if the
    capture had them) and writes PROFILE: per kernel and per op class the device time and share (and DRAM traffic)."""
    import csv  # pylint: disable=import-outside-toplevel
    from collections import OrderedDict  # pylint: disable=import-outside-toplevel
    from bnneon_b200 import pkgread, synth  # pylint: disable=import-outside-toplevel
    launches = OrderedDict()
    hdr = None
    with open(csv_path, encoding="utf-8", errors="replace") as f:
        for r in csv.reader(f):
            if r and r[0] == "ID":
                hdr = r
                continue
            if not hdr or len(r) != len(hdr):
                continue
            d = dict(zip(hdr, r))
            e = launches.setdefault(int(d["ID"]), {"name": d["Kernel Name"].split("(")[0].replace("void ", "").strip()})
            v, u, name = float(d["Metric Value"].replace(",", "")), d["Metric Unit"], d["Metric Name"]
            if name == "gpu__time_duration.sum":
                e["us"] = v * {"ns": 1e-3, "nsecond": 1e-3, "us": 1.0, "usecond": 1.0, "ms": 1e3, "msecond": 1e3,
                              "s": 1e6, "second": 1e6}[u]
            elif name.startswith("dram__bytes"):
                e["bytes"] = e.get("bytes", 0.0) + v * {"byte": 1, "Kbyte": 1e3, "KB": 1e3, "Mbyte": 1e6, "MB": 1e6,
                                                         "Gbyte": 1e9, "GB": 1e9}[u]
    lst = list(launches.values())
    td = tempfile.mkdtemp()
    pkg = os.path.join(td, "v24_full.bnpk")
    synth.make_package(pkg, seed=0)
    ops, _ = pkgread.read_ops(pkg)
    cls, i = OrderedDict(), 0
    for code, _, _, _ in ops:  # assign the launches to the ops in order
        c = cls.setdefault(OPCODE_NAMES.get(code, str(code)), {"us": 0.0, "bytes": 0.0, "ops": 0, "launches": 0})
        c["ops"] += 1
        for kname in OP_KERNELS[code]:
            if (code == 25 or kname == "k_quant") and (i >= len(lst) or not lst[i]["name"].startswith(kname)):
                continue  # work done inside the launch of the op before (a fused SE gate or quantizer)
            if i >= len(lst) or not lst[i]["name"].startswith(kname):
                raise SystemExit(f"launch {i} ({lst[i]['name'] if i < len(lst) else 'none'}) is not {kname}")
            c["us"] += lst[i]["us"]
            c["bytes"] += lst[i].get("bytes", 0.0)
            c["launches"] += 1
            i += 1
    tot = sum(e["us"] for e in lst)
    kern = OrderedDict()
    for e in lst:
        k = kern.setdefault(e["name"], [0, 0.0, 0.0])
        k[0] += 1
        k[1] += e["us"]
        k[2] += e.get("bytes", 0.0)
    dram = any("bytes" in e for e in lst)
    out = [f"# Launch list: full v2.4 int8 package, batch {batch}, one step ({len(lst)} launches)", "",
           "Command (GPU box, after the same command line without `ncu` exited 0):", "",
           "    python bench.py --ncu --warmup 3 && \\",
           "    " + NCU_CMD.format(skip=3 * len(lst), count=len(lst)), "",
           "then `python bench.py --ncu-summary <out>/launches.csv` wrote this file. Per-launch times are",
           "serialised and cold-cache (ncu flushes caches between launches); the shares are what compare with the",
           "bench's per-op CUDA-event times.", "",
           "| kernel | launches | total µs | share |" + (" DRAM MB | GB/s |" if dram else ""),
           "|---|---:|---:|---:|" + ("---:|---:|" if dram else "")]
    for k, (n, us, by) in sorted(kern.items(), key=lambda kv: -kv[1][1]):
        out.append(f"| {k} | {n} | {us:.1f} | {100 * us / tot:.1f}% |" +
                   (f" {by / 1e6:.1f} | {by / us / 1e3:.0f} |" if dram else ""))
    out += [f"| **total** | {len(lst)} | {tot:.1f} | |" + (" | |" if dram else ""), "",
            "Per op class (the package's ops):", "",
            "| op class | ops | launches | total µs | share |", "|---|---:|---:|---:|---:|"]
    for k, c in sorted(cls.items(), key=lambda kv: -kv[1]["us"]):
        out.append(f"| {k} | {c['ops']} | {c['launches']} | {c['us']:.1f} | {100 * c['us'] / tot:.1f}% |")
    out.append("")
    with open(PROFILE, "w", encoding="utf-8") as f:
        f.write("\n".join(out))
    print(f"wrote {PROFILE}")


TRAFFIC = os.path.join(REPO, "profiles", "traffic_pw_s8n_v24_int8_b64.md")


def profile_traffic(cls_name, alg_bytes_per_op):
    """DRAM bytes per op of an op class, from the committed one-op capture (profiles/traffic_*: the DRAM bytes of one
    representative op's launches at a small batch against that op's algorithmic bytes) scaled to the class's
    algorithmic bytes per op: (bytes, ratio, what), or (None, None, None) if there is no capture for the class."""
    try:
        with open(TRAFFIC, encoding="utf-8") as f:
            txt = f.read()
        blk = json.loads(txt.split("```json", 1)[1].split("```", 1)[0])
        if blk["class"] != cls_name:
            return None, None, None
        ratio = blk["dram_bytes"] / blk["algorithmic_bytes"]
        return round(ratio * alg_bytes_per_op), round(ratio, 3), blk["what"]
    except (OSError, IndexError, KeyError, ValueError):
        return None, None, None


def c1_gemm(m, torch, stream, peak_bf16):
    """Config 1 timed: one int8 GEMM M 4096 x K 256 x N 512 on given int8 rows through
    bnn_pw_s8_gemm, 50 launches back to back, CUDA events on their stream; fp32 outputs (the harness requant is in
    the parity test). int8 ops = 2 M N K per launch."""
    from bnneon_b200 import synth  # pylint: disable=import-outside-toplevel
    Mr, K, N = 4096, 256, 512
    a = np.random.default_rng(1).integers(-127, 128, (Mr, K)).astype(np.int8)
    w = np.random.default_rng(2).normal(0.0, 0.02, (N, K)).astype(np.float32)
    lw = synth._Int8Lowering([])  # pylint: disable=protected-access
    tl, (n, k, kp, np_) = lw.s8("c1", w, np.zeros(N, np.float32))
    wq, sw, cs, bb = [lw.tensors[t][1] for t in tl]
    h = m.h.bnn_pw_s8_new(n, k, kp, np_, wq.ctypes.data, sw.ctypes.data, cs.ctypes.data, bb.ctypes.data, Mr)
    if not h:
        return None
    try:
        q = torch.from_numpy(a).cuda()
        sa = torch.full((Mr,), 0.05, dtype=torch.float32, device="cuda")
        za = torch.zeros(Mr, dtype=torch.int32, device="cuda")
        out = torch.empty(Mr * np_, dtype=torch.float32, device="cuda")

        def run():
            return m.h.bnn_pw_s8_gemm(h, 1, Mr, q.data_ptr(), kp, sa.data_ptr(), za.data_ptr(), 0, out.data_ptr(),
                                      Mr * np_, np_, 0, 0, None, 0, 0, 0, 0, stream.cuda_stream)
        for _ in range(5):
            run()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 50
        e0.record(stream)
        for _ in range(reps):
            run()
        e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
    finally:
        m.h.bnn_pw_s8_free(h)
    ops = 2.0 * Mr * N * K
    peak = 2.0 * peak_bf16
    nbytes = Mr * K + N * K + 3 * 4 * N + Mr * N * 4
    return {"shape": "M 4096 x K 256 x N 512, int8 rows given, fp32 out", "us_per_launch": round(us, 2),
            "tops": round(ops / (us * 1e-6) / 1e12, 1), "int8_peak_tops": round(peak, 1),
            "frac_of_int8_peak": round(ops / (us * 1e-6) / 1e12 / peak, 4),
            "algorithmic_bytes": nbytes, "GB/s": round(nbytes / (us * 1e-6) / 1e9, 1),
            "note": "int8 peak = 2 x the measured dense bf16 GEMM rate (MEASURED_PEAKS.json bf16_tflops; B200 runs "
                    "dense int8 at twice bf16); the shape is HBM / latency bound (AI 112 op/B), so TOPS is far below "
                    "the int8 ridge"}


PROTO_C4 = dict(batch=512, cells=64, channels=1536, classes=14795, ppc=4)


def int8_peak(torch):
    """Dense int8 tensor-core throughput measured here: torch._int_mm (cuBLASLt, int8 x int8 -> int32) on 8192^3, best
    of 10 launches (CUDA events); None if the library call is unavailable."""
    try:
        a = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda")
        b = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda").t()
        for _ in range(3):
            torch._int_mm(a, b)  # pylint: disable=protected-access
        best = None
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)  # pylint: disable=protected-access
            e1.record()
            e1.synchronize()
            t = e0.elapsed_time(e1)
            best = t if best is None else min(best, t)
        return 2.0 * 8192 ** 3 / (best * 1e-3) / 1e12
    except (RuntimeError, AttributeError):
        return None


def proto_setup(h, torch, batch, seed=2024):
    """The Perch v2 prototype head (config 4: 64 cells x 1536 channels -> 14795 classes x 4 prototypes) as a
    bnn_proto_s8 op for `batch` windows, with seeded N(0, 1) cells resident on the device."""
    from bnneon_b200 import synth  # pylint: disable=import-outside-toplevel
    c = PROTO_C4
    head = synth.proto_head(seed, c["cells"], c["channels"], c["classes"], c["ppc"], 1e-6)
    qp, sw, n4, rows = synth.pack_proto_s8(head["P"])
    del head["P"]
    cw, cb = np.ascontiguousarray(head["cw"]), np.ascontiguousarray(head["cb"])
    host = {"rows": rows, "sw": sw, "cw": cw, "cb": cb}
    n = c["classes"] * c["ppc"]
    np_, kp = rows.shape
    op = h.bnn_proto_s8_new(n, c["channels"], kp, np_, qp.ctypes.data, sw.ctypes.data, n4.ctypes.data, cw.ctypes.data,
                            cb.ctypes.data, c["classes"], c["ppc"], 1e-6, c["cells"], batch)
    if not op:
        raise RuntimeError(h.bnn_last_error().decode())
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((batch, c["cells"], c["channels"]), generator=g, device="cuda", dtype=torch.float32)
    lg = torch.empty((batch, c["classes"]), dtype=torch.float32, device="cuda")
    cm = torch.empty((batch, np_), dtype=torch.float32, device="cuda")
    st = torch.empty(batch, dtype=torch.int32, device="cuda")

    def run(stream_ptr):
        return h.bnn_proto_s8_run(op, batch, x.data_ptr(), c["cells"] * c["channels"], c["channels"], lg.data_ptr(),
                                  c["classes"], cm.data_ptr(), np_, st.data_ptr(), stream_ptr)
    return op, run, (x, lg, cm, st, host), np_, kp


def proto_cpu_baseline(keep, n, seconds=15.0):
    """The oracle port of PROTO_S8 (oracle/oracle_proto.c, restating src/proto_s8n.c and pc_proto_logits) on this
    host's cores: windows of the same cells, one window per thread; a first round of one window per thread, then, if
    that was short, one sample of whole rounds sized to about half of `seconds`."""
    from oracle import oracle  # pylint: disable=import-outside-toplevel
    c = PROTO_C4
    x_dev, host = keep[0], keep[4]
    threads = os.cpu_count() or 1
    lib = oracle.lib()
    def run(n_win):
        x = np.ascontiguousarray(x_dev[:n_win].cpu().numpy())
        lg = np.empty((n_win, c["classes"]), np.float32)
        t0 = time.perf_counter()
        lib.bnno_proto_s8_many(n_win, threads, oracle.ptr(x), c["cells"] * c["channels"], c["cells"], c["channels"],
                               c["channels"], 1e-6, oracle.ptr(host["rows"]), oracle.ptr(host["sw"]),
                               host["rows"].shape[0], host["rows"].shape[1], oracle.ptr(host["cw"]),
                               oracle.ptr(host["cb"]), c["classes"], c["ppc"], oracle.ptr(lg))
        return time.perf_counter() - t0
    n_win = min(threads, n)
    dt = run(n_win)
    if dt < seconds / 3:  # one more, longer sample: whole rounds of one window per thread
        n_win = min(n, threads * max(1, int(seconds / 2 / dt)))
        dt = run(n_win)
    return {"value": round(n_win / dt, 3), "unit": "windows/s", "cores": threads, "kind": "port",
            "sample": f"{n_win} windows of the same head and cells ({dt:.1f} s, oracle/oracle_proto.c, one thread per "
                      f"window)"}


def proto_head_c4(h, torch, stream, peak_bf16, cpu=True):
    """Config 4's int8 head timed: PROTO_S8 (per-cell quantizer, tcgen05 column-max GEMM, logits) on 512 windows
    through bnn_proto_s8_run, inputs resident, 20 runs back to back after 3 warm-ups, CUDA events on their stream.
    The GEMM is tensor-core bound (M 32768 cells x N 59180 x K 1536: 5.96 T int8 ops per run)."""
    c = PROTO_C4
    B = c["batch"]
    op, run, keep, np_, kp = proto_setup(h, torch, B)
    try:
        sp = stream.cuda_stream
        for _ in range(3):
            assert run(sp) == 0
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        e0.record(stream)
        for _ in range(reps):
            run(sp)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        err = h.bnn_proto_s8_error(op)
        base = proto_cpu_baseline(keep, B) if cpu else None
    finally:
        h.bnn_proto_s8_free(op)
        del keep
    n = c["classes"] * c["ppc"]
    ops = 2.0 * B * c["cells"] * n * c["channels"]
    tops = ops / (ms * 1e-3) / 1e12
    meas = int8_peak(torch)
    peak = meas if meas else 2.0 * peak_bf16
    return {"shape": f"{B} windows x {c['cells']} cells x K {c['channels']} -> {n} prototypes ({c['classes']} classes "
                     f"x {c['ppc']}), fp32 cells in, logits out", "ms_per_run": round(ms, 4),
            "windows_per_s": round(B / (ms * 1e-3), 1), "int8_ops_per_run": ops, "tops": round(tops, 1),
            "roofline": {"bound": "tensor", "achieved": round(tops, 1), "peak": round(peak, 1), "unit": "TOP/s",
                         "frac": round(tops / peak, 4),
                         "peak_source": "measured here: torch._int_mm (cuBLASLt int8) 8192^3, best of 10" if meas
                         else "2 x MEASURED_PEAKS.json bf16_tflops (torch._int_mm unavailable)"},
            "gemm_error_word": err, "cpu_baseline": base,
            "note": "time = the whole op (quantizer + GEMM + logits); ops = the GEMM's 2 M N K"}


def logmel_perch(h, torch, stream, hbm_peak, cpu=True, batch=512):
    """The Perch-like log-mel front end (FE_LOGMEL: 160000 samples at 32 kHz, 640-sample frames, hop 320, 1024-point
    FFT, 128 mel bins -> 499 x 128) on `batch` windows through bnn_logmel_run, inputs resident, CUDA events over 20
    runs after 3 warm-ups; CPU baseline: the oracle port on this host's cores."""
    from bnneon_b200 import synth  # pylint: disable=import-outside-toplevel
    p = synth.PERCH_FE
    fe = synth.logmel_frontend(p["nsamp"], p["frame"], p["hop"], p["pad"], p["nfft"], p["nmel"], p["fmin"], p["fmax"],
                               p["floor"], p["scale"])
    mel = np.ascontiguousarray(fe["mel"])
    op = h.bnn_logmel_new(p["nsamp"], p["frame"], p["hop"], p["pad"], p["nfft"], p["nmel"], fe["window"].ctypes.data,
                          mel.ctypes.data, p["floor"], p["scale"])
    if not op:
        return None
    try:
        nfr = h.bnn_logmel_frames(op)
        g = torch.Generator(device="cuda").manual_seed(7)
        x = (0.1 * torch.randn((batch, p["nsamp"]), generator=g, device="cuda")).float()
        out = torch.empty((batch, nfr * p["nmel"]), dtype=torch.float32, device="cuda")
        sp = stream.cuda_stream

        def run():
            return h.bnn_logmel_run(op, batch, x.data_ptr(), p["nsamp"], out.data_ptr(), nfr * p["nmel"], sp)
        for _ in range(3):
            assert run() == 0
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(20):
            run()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / 20
        base = None
        if cpu:
            from oracle import oracle  # pylint: disable=import-outside-toplevel
            threads = os.cpu_count() or 1
            xs = x[:threads].cpu().numpy()
            t0 = time.perf_counter()
            import concurrent.futures  # pylint: disable=import-outside-toplevel
            with concurrent.futures.ThreadPoolExecutor(threads) as ex:  # the oracle releases the GIL in C
                list(ex.map(lambda w: oracle.logmel(xs[w:w + 1], p["frame"], p["hop"], p["pad"], p["nfft"],
                                                    fe["window"], mel, p["floor"], p["scale"]), range(len(xs))))
            dt = time.perf_counter() - t0
            base = {"value": round(len(xs) / dt, 2), "unit": "windows/s", "cores": threads, "kind": "port",
                    "sample": f"{len(xs)} windows, one per thread (oracle/oracle_ops.c bnno_logmel_run), {dt:.2f} s"}
    finally:
        h.bnn_logmel_free(op)
    nbytes = batch * (p["nsamp"] + nfr * p["nmel"]) * 4
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"shape": f"{batch} windows x {p['nsamp']} samples -> {nfr} x {p['nmel']} (frame {p['frame']}, hop "
                     f"{p['hop']}, nfft {p['nfft']})", "ms_per_run": round(ms, 4),
            "windows_per_s": round(batch / (ms * 1e-3), 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(gbs / hbm_peak, 4),
                         "note": "algorithmic bytes = samples in + spectrogram out; the shared-memory FFT passes, "
                                 "not HBM, bound this kernel"},
            "cpu_baseline": base}


def hfma2_peak(h, torch, stream):
    """The fp16 FMA pipe's throughput measured here (bnn_cuda_peak_hfma2: 148 x 8 CTAs of 256 threads, 8 independent
    fma.rn.f16x2 chains each), TFLOP/s: the roofline of the neon-fp16 path's CUDA-core kernels."""
    word = torch.zeros(4, dtype=torch.int32, device="cuda")
    blocks, iters, sp = 148 * 8, 20000, stream.cuda_stream
    for _ in range(2):
        assert h.bnn_cuda_peak_hfma2(blocks, iters, word.data_ptr(), sp) == 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(5):
        h.bnn_cuda_peak_hfma2(blocks, iters, word.data_ptr(), sp)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / 5
    return 2.0 * blocks * 256 * iters * 16 / (ms * 1e-3) / 1e12


def fp16_package_leg(torch, stream, pkg, pcm, batch, steps, cpu, workload, parity):
    """One neon-fp16 package on `batch` windows: device-resident windows/s (bnn_infer_device, CUDA events over `steps`
    steps after 3 warm-ups), end to end through bnn_infer_batch with pinned host buffers, the per-op-class device
    time, and the fp16 GEMMs' FLOP/s against the measured fp16 FMA pipe peak. Every kernel is bit-exact against the
    oracle (the reference's fp16 FMA chains on CUDA cores; the tensor cores cannot reproduce them)."""
    from bnneon_b200 import Model, pkgread, synth  # pylint: disable=import-outside-toplevel
    nsamp = pcm.shape[1]
    m = Model(pkg, mode=3, batch=batch)
    try:
        nc, ne = m.info.n_classes, m.info.emb_dim
        d_pcm = torch.from_numpy(pcm).cuda()
        d_out = torch.empty((batch, nc), dtype=torch.float32, device="cuda")
        d_emb = torch.empty((batch, ne), dtype=torch.float32, device="cuda")
        sp = stream.cuda_stream

        def run():
            m.infer_device(batch, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr(), sp)
        for _ in range(3):
            run()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            run()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / steps
        # end to end
        h_pcm = torch.from_numpy(pcm).pin_memory()
        h_out = torch.empty((batch, nc), dtype=torch.float32).pin_memory()
        h_emb = torch.empty((batch, ne), dtype=torch.float32).pin_memory()
        m.infer_batch(h_pcm.numpy(), h_out.numpy(), h_emb.numpy())
        t0 = time.perf_counter()
        for _ in range(3):
            m.infer_batch(h_pcm.numpy(), h_out.numpy(), h_emb.numpy())
        e2e_ms = (time.perf_counter() - t0) * 1e3 / 3
        stream.synchronize()
        timed_out = {"bnn_infer_batch": (h_out.numpy().copy(), h_emb.numpy().copy()),
                     "bnn_infer_device": (d_out.cpu().numpy(), d_emb.cpu().numpy())}
        # per-op classes
        ops, _ = pkgread.read_ops(pkg, synth.PATH_F16)
        m.h.bnn_profile_begin(m.ctx)
        for _ in range(2):
            run()
            m.h.bnn_profile_collect(m.ctx)
        m.h.bnn_profile_end(m.ctx)
        cls = {}
        for i, (code, _, _, p) in enumerate(ops):
            c = cls.setdefault(pkgread.NAMES.get(code, str(code)).lower(), {"ms": 0.0, "flop": 0.0, "ops": 0})
            c["ms"] += m.h.bnn_profile_op_ms(m.ctx, i) / 2
            c["ops"] += 1
            if code == 0x103:
                c["flop"] += 2.0 * batch * p[4] * p[2] * p[3]
        launches = m.launches_per_batch
        tensor = fp16_tensor_mode(m, torch, stream, run, steps, batch, ops, h_pcm, h_out, h_emb, timed_out)
    finally:
        m.close()
    peak = hfma2_peak(m.h, torch, stream)
    pw = cls["pw_f16"]
    tflops = pw["flop"] / (pw["ms"] * 1e-3) / 1e12
    base = None
    if cpu:
        cores = os.cpu_count() or 1
        n = min(batch, cores)
        kind, crun, what = cpu_runner(pkg, mode=3)
        t0 = time.perf_counter()
        crun(pcm[:n], cores)
        dt = time.perf_counter() - t0
        base = {"value": round(n / dt, 3), "unit": "windows/s", "cores": cores, "kind": kind,
                "sample": f"{n} windows, one per thread, {dt:.1f} s: {what} (every fp16 operation emulated exactly "
                          f"in software)"}
    checked = (parity_check(pkg, pcm, timed_out, chunk_boundary_sample(batch, batch, 4), synth.PATH_F16,
                            os.cpu_count() or 1) if cpu else None)
    total = sum(v["ms"] for v in cls.values())
    return {"workload": workload,
            "batch": batch, "ms_per_step": round(ms, 3), "windows_per_s": round(batch / (ms * 1e-3), 1),
            "e2e": {"value": round(batch / (e2e_ms * 1e-3), 1), "unit": "windows/s",
                    "h2d_bytes_per_step": batch * nsamp * 4, "d2h_bytes_per_step": batch * (nc + ne) * 4,
                    "path": "bnn_infer_batch (C ABI), pinned host buffers, wall clock"},
            "gpu_launches_per_step": launches,
            "roofline": {"bound": "fp16 FMA pipe (CUDA cores)", "kernel": f"pw_f16 ({pw['ops']} GEMMs per step)",
                         "achieved": round(tflops, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(tflops / peak, 4),
                         "peak_source": "measured here: bnn_cuda_peak_hfma2 (fma.rn.f16x2 chains on every SM)",
                         "note": "achieved = 2 M K N of the 1x1 convs (Kp, Np as packed) / their CUDA-event time"},
            "ops": {k: {"ms": round(v["ms"], 4), "share": round(v["ms"] / total, 4), "ops": v["ops"]}
                    for k, v in sorted(cls.items(), key=lambda kv: -kv[1]["ms"])},
            "parity": parity, "parity_checked": checked, "cpu_baseline": base, "tensor_mode": tensor}


def sqnr_db(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(10 * np.log10(np.sum(want ** 2) / max(np.sum((got - want) ** 2), 1e-300)))


def fp16_tensor_mode(m, torch, stream, run, steps, batch, ops, h_pcm, h_out, h_emb, exact):
    """The same package in the tensor mode (bnn_set_fp16_tensor: the 1x1 convs as tcgen05 kind::f16 GEMMs with fp32
    accumulators; within a tolerance of the reference, tests/test_gpu_f16_tensor.py): device and end-to-end
    windows/s, the 1x1 convs' device time, and the SQNR of its timed outputs against the bit-exact mode's on sampled
    windows. Leaves the context in the bit-exact mode."""
    from bnneon_b200 import pkgread  # pylint: disable=import-outside-toplevel
    m.set_fp16_tensor(True)
    try:
        for _ in range(3):
            run()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            run()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / steps
        m.infer_batch(h_pcm.numpy(), h_out.numpy(), h_emb.numpy())
        t0 = time.perf_counter()
        for _ in range(3):
            m.infer_batch(h_pcm.numpy(), h_out.numpy(), h_emb.numpy())
        e2e_ms = (time.perf_counter() - t0) * 1e3 / 3
        got, gemb = h_out.numpy().copy(), h_emb.numpy().copy()
        m.h.bnn_profile_begin(m.ctx)
        for _ in range(2):
            run()
            m.h.bnn_profile_collect(m.ctx)
        m.h.bnn_profile_end(m.ctx)
        pw_ms = sum(m.h.bnn_profile_op_ms(m.ctx, i) / 2 for i, (code, _, _, _) in enumerate(ops)
                    if pkgread.NAMES.get(code) == "PW_F16")
    finally:
        m.set_fp16_tensor(False)
    want, wemb = exact["bnn_infer_batch"]
    idx = chunk_boundary_sample(batch, batch, 16)
    return {"ms_per_step": round(ms, 3), "windows_per_s": round(batch / (ms * 1e-3), 1),
            "e2e": {"value": round(batch / (e2e_ms * 1e-3), 1), "unit": "windows/s"},
            "pw_f16_ms": round(pw_ms, 4),
            "min_sqnr_db_vs_bit_exact": {"logits": round(min(sqnr_db(got[w], want[w]) for w in idx), 1),
                                         "embedding": round(min(sqnr_db(gemb[w], wemb[w]) for w in idx), 1),
                                         "windows": len(idx)},
            "note": "bnn_set_fp16_tensor(ctx, 1): the 1x1 convs on tcgen05 kind::f16 with fp32 accumulation instead "
                    "of the reference's fp16 FMA chains; parity by tolerance (tests/test_gpu_f16_tensor.py)"}


def v24_fp16_c3(torch, stream, batch=1024, steps=10, cpu=True):
    """Config 3: the v2.4-architecture neon-fp16 package (the reference compiler's bytes for the same synthetic IR)
    on `batch` windows."""
    from bnneon_b200 import synth  # pylint: disable=import-outside-toplevel
    pkg = os.path.join(tempfile.mkdtemp(), "v24_full_f16.bnpk")
    synth.make_package(pkg, seed=0, path=synth.PATH_F16)
    return fp16_package_leg(
        torch, stream, pkg, synth.audio(batch, seed=4000), batch, steps, cpu,
        "BirdNET-v2.4-architecture neon-fp16 package (config 3): 144000-sample windows, fp16 activations and weights, "
        "6522-class fp16 head",
        "bit-exact against the oracle (tests/test_gpu_f16.py); the oracle within 50 dB SQNR of a float64 model "
        "(tests/test_f16_cpu.py)")


def perch_c4(torch, stream, batch=512, steps=5, cpu=True):
    """Config 4: a Perch-v2-architecture package, neon-fp16 body + the int8 SDOT prototype head (bnc.py compile
    --paths neon-fp16 --proto-s8), 160000-sample windows at 32 kHz, 59180 prototypes, on `batch` windows."""
    from bnneon_b200 import synth  # pylint: disable=import-outside-toplevel
    pkg = os.path.join(tempfile.mkdtemp(), "perch_v2_f16s8.bnpk")
    _, _, ns = synth.make_perch_package(pkg, seed=0)
    pcm = synth.audio(batch, seed=4100, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
    return fp16_package_leg(
        torch, stream, pkg, pcm, batch, steps, cpu,
        "Perch-v2-architecture neon-fp16 package with the int8 prototype head (config 4): 160000-sample windows, "
        "log-mel front end, fp32 stem, 26 fp16 MBConv blocks, 14795 x 4 int8 prototypes on 64 cells, 1536-d embedding",
        "bit-exact against the oracle (tests/test_gpu_perch.py); the oracle within 50 dB SQNR of a float64 model on "
        "the embedding (tests/test_perch_cpu.py)")


def perch_int8(torch, stream, batch=512, steps=5, cpu=True):
    """The Perch-v2-architecture model on the neon-int8 path (the reference compiler's default int8 policy; the
    reference ships perch_v2-neon-int8.bnpk): device-resident and end-to-end windows/s on `batch` windows, per-op-class
    device time, the timed outputs of sampled windows against the reference runtime (oracle/_ref) bit for bit."""
    from bnneon_b200 import Model, pkgread, synth  # pylint: disable=import-outside-toplevel
    pkg = os.path.join(tempfile.mkdtemp(), "perch_v2_int8.bnpk")
    _, _, ns = synth.write_perch_int8_package(pkg, synth.perch_ir(0))
    pcm = synth.audio(batch, seed=4300, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
    m = Model(pkg, mode=4, batch=batch)
    try:
        nc, ne = m.info.n_classes, m.info.emb_dim
        d_pcm = torch.from_numpy(pcm).cuda()
        d_out = torch.empty((batch, nc), dtype=torch.float32, device="cuda")
        d_emb = torch.empty((batch, ne), dtype=torch.float32, device="cuda")
        sp = stream.cuda_stream

        def run():
            m.infer_device(batch, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr(), sp)
        for _ in range(3):
            run()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            run()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / steps
        h_pcm = torch.from_numpy(pcm).pin_memory()
        h_out = torch.empty((batch, nc), dtype=torch.float32).pin_memory()
        h_emb = torch.empty((batch, ne), dtype=torch.float32).pin_memory()
        m.infer_batch(h_pcm.numpy(), h_out.numpy(), h_emb.numpy())
        t0 = time.perf_counter()
        for _ in range(3):
            m.infer_batch(h_pcm.numpy(), h_out.numpy(), h_emb.numpy())
        e2e_ms = (time.perf_counter() - t0) * 1e3 / 3
        stream.synchronize()
        got, gemb = h_out.numpy().copy(), h_emb.numpy().copy()
        ops, _ = pkgread.read_ops(pkg)
        m.h.bnn_profile_begin(m.ctx)
        for _ in range(2):
            run()
            m.h.bnn_profile_collect(m.ctx)
        m.h.bnn_profile_end(m.ctx)
        cls = {}
        for i, (code, _, _, _) in enumerate(ops):
            c = cls.setdefault(pkgread.NAMES.get(code, str(code)).lower(), {"ms": 0.0, "ops": 0})
            c["ms"] += m.h.bnn_profile_op_ms(m.ctx, i) / 2
            c["ops"] += 1
        launches = m.launches_per_batch
    finally:
        m.close()
    base = checked = None
    if cpu:
        cores = os.cpu_count() or 1
        n = min(batch, cores)
        kind, crun, what = cpu_runner(pkg, mode=4)
        t0 = time.perf_counter()
        crun(pcm[:n], cores)
        dt = time.perf_counter() - t0
        base = {"value": round(n / dt, 3), "unit": "windows/s", "cores": cores, "kind": kind,
                "sample": f"{n} windows, one per thread, {dt:.1f} s: {what}"}
        from oracle import ref  # pylint: disable=import-outside-toplevel
        idx = chunk_boundary_sample(batch, batch, 4)
        want, wemb, rc = ref.run_many(pkg, 4, np.ascontiguousarray(pcm[idx]), threads=min(len(idx), cores))
        bad = int(sum(not (np.array_equal(got[w].view(np.int32), want[j].view(np.int32)) and
                           np.array_equal(gemb[w].view(np.int32), wemb[j].view(np.int32))) for j, w in enumerate(idx)))
        checked = {"windows": len(idx), "calls": ["bnn_infer_batch"], "mismatched": bad, "bit_exact": bad == 0,
                   "reference_rc": int(np.abs(rc).sum()),
                   "against": "oracle/_ref (the reference's own C runtime built for this host), logits and embeddings"}
    total = sum(v["ms"] for v in cls.values())
    return {"workload": "Perch-v2-architecture neon-int8 package (the reference compiler's default int8 policy): "
                        "160000-sample windows, log-mel front end, fp32 stem, 26 MBConv blocks with int8 expansions "
                        "and fp32 SE-gated projections, int8 1536-channel top conv, 14795 x 4 int8 prototypes",
            "batch": batch, "ms_per_step": round(ms, 3), "windows_per_s": round(batch / (ms * 1e-3), 1),
            "e2e": {"value": round(batch / (e2e_ms * 1e-3), 1), "unit": "windows/s",
                    "h2d_bytes_per_step": batch * ns * 4, "d2h_bytes_per_step": batch * (nc + ne) * 4,
                    "path": "bnn_infer_batch (C ABI), pinned host buffers, wall clock"},
            "gpu_launches_per_step": launches,
            "ops": {k: {"ms": round(v["ms"], 4), "share": round(v["ms"] / total, 4), "ops": v["ops"]}
                    for k, v in sorted(cls.items(), key=lambda kv: -kv[1]["ms"])},
            "parity_checked": checked, "cpu_baseline": base}


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json"), encoding="utf-8") as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


class Clocks:
    """SM clock and throttle-reason samples (NVML, every 10 ms) while the timed region runs; nvidia-smi if NVML is
    missing. The first sample is taken before the timed region starts."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, index):
        self.index, self.rows, self.proc, self.nv, self.stop = index, [], None, None, threading.Event()

    def _handle(self):
        import pynvml  # pylint: disable=import-outside-toplevel
        pynvml.nvmlInit()
        try:
            import torch  # pylint: disable=import-outside-toplevel
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:  # pylint: disable=broad-except
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _sample_nvml(self, nv, h):
        while True:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((float(sm), float(mx), int(rs)))
            except Exception:  # pylint: disable=broad-except
                pass
            if self.stop.wait(0.01):
                break

    def __enter__(self):
        try:
            nv, h = self._handle()
            self.nv = nv
            self.th = threading.Thread(target=self._sample_nvml, args=(nv, h), daemon=True)
            self.th.start()
            t = time.time()
            while not self.rows and time.time() - t < 2:
                time.sleep(0.005)
            return self
        except Exception:  # pylint: disable=broad-except
            self.nv = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read_smi, daemon=True)
            self.th.start()
            t = time.time()
            while not self.rows and time.time() - t < 3:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        return self

    def _read_smi(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.proc.stdout:
            r = [x.strip() for x in line.split(",")]
            try:
                mask = sum(self.REASONS[n] for i, n in enumerate(names) if r[4 + i].lower().startswith("active"))
                self.rows.append((float(r[0]), float(r[1]), mask))
            except (ValueError, IndexError):
                continue

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if getattr(self, "th", None):
            self.th.join(timeout=2)

    def summary(self):
        sm = [r[0] for r in self.rows]
        reasons = sorted({n for r in self.rows for n, bit in self.REASONS.items() if r[2] & bit})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": self.rows[-1][1] if self.rows else None,
                "reasons": reasons, "samples": len(sm), "source": "nvml" if self.nv else "nvidia-smi"}


REF_SAMPLE = ("the reference's own C runtime (its src/*.c, unmodified) compiled for this x86 host by oracle/ref.mk: "
              "NEON intrinsics through a scalar stand-in written from the Arm ARM, auto-vectorized by GCC; one "
              "single-threaded bnn_init context per host thread (windows are independent)")
PORT_SAMPLE = "oracle/liboracle.so, the C restatement of the reference's neon-int8 path"


def cpu_runner(pkg, mode=4):
    """The CPU implementation the baselines time: the reference build (oracle/_ref) when present, else the port.
    Returns (kind, run(pcm, threads), description)."""
    from oracle import oracle, ref  # pylint: disable=import-outside-toplevel
    if ref.available():
        def run(x, threads):
            _, _, rc = ref.run_many(pkg, mode, x, threads=threads)
            if rc.any():
                raise RuntimeError("reference build: a window failed")
        return "reference", run, REF_SAMPLE

    def run_port(x, threads):
        oracle.run_many(pkg, x, threads=threads, path_name="neon-int8" if mode == 4 else "neon-fp16")
    return "port", run_port, PORT_SAMPLE


def cpu_baseline(pkg, pcm, seconds=12.0):
    """The reference's CPU implementation on all host cores over a bounded sample: windows/s."""
    cores = os.cpu_count() or 1
    kind, run, what = cpu_runner(pkg)
    t = time.time()
    run(pcm[:cores], cores)  # calibration round: one window per core
    per_round = time.time() - t
    rounds = max(1, min(16, int(seconds / max(per_round, 1e-3))))
    n = min(pcm.shape[0], cores * rounds)
    reps = max(1, (cores * rounds) // n)
    t = time.time()
    for _ in range(reps):
        run(pcm[:n], cores)
    dt = time.time() - t
    return {"value": round(n * reps / dt, 3), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{n * reps} windows ({reps} x {n}) of the same synthetic batch on {cores} threads, {dt:.1f} s: "
                      f"{what}"}


def parity_check(pkg, pcm, results, idx, path_name, threads):
    """The checker, after the timed regions: the outputs the timed calls produced for the windows `idx` of the timed
    batch against the CPU oracle (oracle/liboracle.so), bit for bit. results = {call name: (out, emb)}."""
    from oracle import oracle  # pylint: disable=import-outside-toplevel
    want, wemb = oracle.run_many(pkg, np.ascontiguousarray(pcm[idx]), threads=max(1, min(threads, len(idx))),
                                 path_name=path_name)
    bad = 0
    for out, emb in results.values():
        for j, w in enumerate(idx):
            same = np.array_equal(np.asarray(out[w]).view(np.int32), want[j].view(np.int32))
            if emb is not None:
                same = same and np.array_equal(np.asarray(emb[w]).view(np.int32), wemb[j].view(np.int32))
            bad += 0 if same else 1
    return {"windows": len(idx), "calls": sorted(results), "mismatched": bad, "bit_exact": bad == 0,
            "against": "oracle/liboracle.so (CPU restatement of the reference path), logits and embeddings"}


def chunk_boundary_sample(n, batch, k):
    """k windows of a batch of n: the first and last, both sides of the first chunk boundary of bnn_infer_batch (a
    quarter of the batch, rounded up to 8) and evenly spaced ones"""
    c = (min(n, batch) // 4 + 7) // 8 * 8 if min(n, batch) >= 64 else n
    idx = {0, n - 1, min(c, n - 1), max(c - 1, 0)}
    for w in np.linspace(0, n - 1, k).astype(int):
        if len(idx) >= k:
            break
        idx.add(int(w))
    return np.array(sorted(idx))


def reference_arm(args, rank):
    if rank != 0:
        return
    from bnneon_b200 import synth  # pylint: disable=import-outside-toplevel
    cores = os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as td:
        pkg = os.path.join(td, "v24_full.bnpk")
        synth.make_package(pkg, seed=0)
        kind, run, what = cpu_runner(pkg)
        n = 2 * cores  # a bounded sample per step
        pcm = synth.audio(n, seed=100)
        for _ in range(args.warmup):
            run(pcm, cores)
        t = time.time()
        for _ in range(args.steps):
            run(pcm, cores)
        dt = time.time() - t
    value = n * args.steps / dt
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "batch_per_gpu": args.batch, "cpu_sample_windows_per_step": n},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": f"{n} windows per step on {cores} threads: {what}"},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu-summary", metavar="CSV",
                    help="write profiles/launch_list_v24_int8_b256.md from an ncu launch-list CSV (no GPU needed)")
    ap.add_argument("--no-proto", action="store_true",
                    help="skip the secondary lines (C4 int8 head, Perch log-mel front end, C3 fp16 package)")
    ap.add_argument("--proto-ncu", type=int, metavar="B", default=0,
                    help="for profiler captures: the prototype head on B windows, 3 warm-ups + 1 run, no timing")
    ap.add_argument("--logmel-ncu", type=int, metavar="B", default=0,
                    help="for profiler captures: the Perch-like log-mel front end on B windows, 3 warm-ups + 1 run")
    ap.add_argument("--f16-ncu", type=int, metavar="B", default=0,
                    help="for profiler captures: the v2.4 neon-fp16 package on B windows, 3 warm-ups + 1 step")
    ap.add_argument("--perch-ncu", type=int, metavar="B", default=0,
                    help="for profiler captures: the Perch-architecture neon-fp16 package on B windows, 3 warm-ups + 1 "
                         "step")
    ap.add_argument("--perch8-ncu", type=int, metavar="B", default=0,
                    help="for profiler captures: the Perch-architecture neon-int8 package on B windows, 4 steps")
    ap.add_argument("--f16-tensor", action="store_true",
                    help="with --f16-ncu / --perch-ncu: the fp16 package in the tensor mode (bnn_set_fp16_tensor)")
    ap.add_argument("--ncu", action="store_true",
                    help="for profiler captures: warm-up steps + one step through bnn_infer_device, no timing, no JSON")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.ncu_summary:
        ncu_summary(args.ncu_summary, args.batch)
        return
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    if args.ncu or args.proto_ncu or args.logmel_ncu or args.f16_ncu or args.perch_ncu or args.perch8_ncu:
        # profiler captures use eager launches: a run that replays the op list from CUDA graphs stopped with a driver
        # LaunchFailed under ncu (the same command exits 0 without ncu)
        os.environ["BNN_GRAPHS"] = "0"

    import torch  # pylint: disable=import-outside-toplevel
    import torch.distributed as dist  # pylint: disable=import-outside-toplevel
    from bnneon_b200 import Model, synth  # pylint: disable=import-outside-toplevel
    import datetime  # pylint: disable=import-outside-toplevel

    torch.cuda.set_device(local)
    os.environ["BNN_DEVICES"] = str(local)
    if args.logmel_ncu:  # the log-mel front end alone, for a profiler; nothing is timed or printed as a result
        from bnneon_b200 import load_library, synth  # pylint: disable=import-outside-toplevel
        h = load_library()
        assert h.bnn_cuda_device_init() == 0
        p = synth.PERCH_FE
        fe = synth.logmel_frontend(p["nsamp"], p["frame"], p["hop"], p["pad"], p["nfft"], p["nmel"], p["fmin"],
                                   p["fmax"], p["floor"], p["scale"])
        mel = np.ascontiguousarray(fe["mel"])
        op = h.bnn_logmel_new(p["nsamp"], p["frame"], p["hop"], p["pad"], p["nfft"], p["nmel"],
                              fe["window"].ctypes.data, mel.ctypes.data, p["floor"], p["scale"])
        nfr, B = h.bnn_logmel_frames(op), args.logmel_ncu
        x = torch.randn((B, p["nsamp"]), device="cuda") * 0.1
        out = torch.empty((B, nfr * p["nmel"]), device="cuda")
        for _ in range(4):
            assert h.bnn_logmel_run(op, B, x.data_ptr(), p["nsamp"], out.data_ptr(), nfr * p["nmel"], None) == 0
        torch.cuda.synchronize()
        h.bnn_logmel_free(op)
        print(f"logmel ncu mode: 4 runs of {B} windows", flush=True)
        return
    if args.f16_ncu or args.perch_ncu or args.perch8_ncu:  # a package alone, for a profiler; nothing is timed
        B = args.f16_ncu or args.perch_ncu or args.perch8_ncu
        td = tempfile.mkdtemp()
        mode = 3
        if args.perch8_ncu:
            pkg = os.path.join(td, "perch_v2_int8.bnpk")
            _, _, ns = synth.write_perch_int8_package(pkg, synth.perch_ir(0))
            pcm = synth.audio(B, seed=4300, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
            mode = 4
        elif args.perch_ncu:
            pkg = os.path.join(td, "perch_v2_f16s8.bnpk")
            _, _, ns = synth.make_perch_package(pkg, seed=0)
            pcm = synth.audio(B, seed=4100, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
        else:
            pkg = os.path.join(td, "v24_full_f16.bnpk")
            synth.make_package(pkg, seed=0, path=synth.PATH_F16)
            pcm = synth.audio(B, seed=4000)
        m = Model(pkg, mode=mode, batch=B, fp16_tensor=True if args.f16_tensor and mode == 3 else None)
        d_pcm = torch.from_numpy(pcm).cuda()
        d_out = torch.empty((B, m.info.n_classes), dtype=torch.float32, device="cuda")
        d_emb = torch.empty((B, m.info.emb_dim), dtype=torch.float32, device="cuda")
        for _ in range(4):
            m.infer_device(B, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr(), None)
        torch.cuda.synchronize()
        print(f"f16 ncu mode: 4 steps of {m.launches_per_batch} launches on {B} windows", flush=True)
        m.close()
        return
    if args.proto_ncu:  # the prototype head alone, for a profiler; nothing is timed or printed as a result
        from bnneon_b200 import load_library  # pylint: disable=import-outside-toplevel
        h = load_library()
        assert h.bnn_cuda_device_init() == 0
        op, run, keep, _, _ = proto_setup(h, torch, args.proto_ncu)
        for _ in range(4):
            assert run(None) == 0
        torch.cuda.synchronize()
        h.bnn_proto_s8_free(op)
        del keep
        print(f"proto ncu mode: 4 runs of {args.proto_ncu} windows", flush=True)
        return
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    B = args.batch
    td = tempfile.mkdtemp()
    pkg = os.path.join(td, "v24_full.bnpk")
    synth.make_package(pkg, seed=0)
    pcm = synth.audio(B, seed=1000 + rank)
    m = Model(pkg, mode=4, batch=B)
    nc, ne = m.info.n_classes, m.info.emb_dim
    stream = torch.cuda.Stream()
    d_pcm = torch.from_numpy(pcm).cuda()
    d_out = torch.empty((B, nc), dtype=torch.float32, device="cuda")
    d_emb = torch.empty((B, ne), dtype=torch.float32, device="cuda")
    sp = stream.cuda_stream

    if args.ncu:  # warm-up + 1 step for a profiler; nothing is timed or printed as a result
        for _ in range(args.warmup + 1):
            m.infer_device(B, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr(), sp)
        stream.synchronize()
        print(f"ncu mode: {args.warmup + 1} steps of {m.launches_per_batch} launches", flush=True)
        m.close()
        return

    # ---- device-resident throughput
    for _ in range(args.warmup):
        m.infer_device(B, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr(), sp)
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = Clocks(local).__enter__()  # sampled through both timed regions (device-resident and end to end)
    ev0.record(stream)
    for _ in range(args.steps):
        m.infer_device(B, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr(), sp)
    ev1.record(stream)
    ev1.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    value = world * B / (ms / 1e3)

    # ---- end to end through bnn_infer_batch: pinned host buffers, copies inside the timed region
    h_pcm = torch.from_numpy(pcm).pin_memory()
    h_out = torch.empty((B, nc), dtype=torch.float32).pin_memory()
    h_emb = torch.empty((B, ne), dtype=torch.float32).pin_memory()
    out_np, emb_np, pcm_np = h_out.numpy(), h_emb.numpy(), h_pcm.numpy()
    for _ in range(2):
        m.infer_batch(pcm_np, out_np, emb_np)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.infer_batch(pcm_np, out_np, emb_np)
    e1.record()
    e1.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / args.steps
    clk.__exit__(None, None, None)
    e2e_ms = max_over_ranks(max(e0.elapsed_time(e1) / args.steps, wall))
    e2e = {"value": round(world * B / (e2e_ms / 1e3), 3), "unit": UNIT, "h2d_bytes_per_step": B * 144000 * 4,
           "d2h_bytes_per_step": B * (nc + ne) * 4, "ms_per_step": round(e2e_ms, 3),
           "path": "bnn_infer_batch (C ABI), pinned host buffers"}

    # ---- the host-to-device copy ceiling: the same 147 MB of pinned PCM per GPU copied by every rank at once with
    # nothing else running (plain cudaMemcpyAsync), max over ranks; e2e cannot beat world * B windows per that time
    copy_ms = []
    for _ in range(6):
        barrier()
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        with torch.cuda.stream(stream):
            d_pcm.copy_(h_pcm, non_blocking=True)
        c1.record(stream)
        c1.synchronize()
        copy_ms.append(c0.elapsed_time(c1))
    cp_ms = max_over_ranks(float(np.median(copy_ms[1:])))
    h2d = B * 144000 * 4
    copy_ceiling = {"h2d_ms_per_gpu": round(cp_ms, 3), "h2d_GBps_per_gpu": round(h2d / (cp_ms / 1e3) / 1e9, 1),
                    "e2e_windows_per_s_ceiling": round(world * B / (cp_ms / 1e3), 1),
                    "e2e_h2d_GBps_per_gpu": round(h2d / (e2e_ms / 1e3) / 1e9, 1),
                    "e2e_frac_of_ceiling": round(cp_ms / e2e_ms, 4),
                    "note": "every rank copies its step's PCM (pinned host -> device, one cudaMemcpyAsync) at the same "
                            "time, nothing else running; max over ranks"}

    # ---- the unchanged per-window call (bnn_infer: one window per call, as BirdNET-Go makes it; the reference's
    # bench/cli.c:203 metric, median ms per window): wall clock per call on rank 0
    lat = None
    if rank == 0:
        lat_ms = []
        for w in range(40 + 200):
            t1 = time.perf_counter()
            m.infer(pcm[w % B])
            if w >= 40:
                lat_ms.append((time.perf_counter() - t1) * 1e3)
        lat = {"p50_ms": round(float(np.percentile(lat_ms, 50)), 4), "p99_ms": round(float(np.percentile(lat_ms, 99)), 4),
               "windows": len(lat_ms), "windows_per_s": round(len(lat_ms) / (sum(lat_ms) / 1e3), 1),
               "path": "bnn_infer (C ABI), one window per call, host buffers, wall clock"}

    # ---- the checker: the timed calls' outputs against the CPU oracle (every window at N = 1, a sample per rank
    # otherwise, so that N processes share the host cores)
    torch.cuda.synchronize()
    idx = np.arange(B) if world == 1 else chunk_boundary_sample(B, B, 16)
    parity = parity_check(pkg, pcm, {"bnn_infer_batch": (out_np, emb_np),
                                     "bnn_infer_device": (d_out.cpu().numpy(), d_emb.cpu().numpy())},
                          idx, synth.PATH, max(1, (os.cpu_count() or 1) // world))
    if world > 1:
        t = torch.tensor([parity["mismatched"], parity["windows"]], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        parity.update({"mismatched": int(t[0].item()), "windows": int(t[1].item()), "bit_exact": int(t[0].item()) == 0,
                       "scope": f"{len(idx)} windows per rank, {world} ranks"})

    # ---- per-op device times (CUDA events around every op on the launching stream)
    from bnneon_b200 import pkgread  # pylint: disable=import-outside-toplevel
    ops, bufs = pkgread.read_ops(pkg)
    m.h.bnn_profile_begin(m.ctx)
    reps = 3
    for _ in range(reps):
        m.infer_device(B, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr(), sp)
        m.h.bnn_profile_collect(m.ctx)
    m.h.bnn_profile_end(m.ctx)
    cls = {}
    for i, (code, bl, _, p) in enumerate(ops):
        t = m.h.bnn_profile_op_ms(m.ctx, i) / reps
        by, wb, macs = op_cost(code, p, bufs, bl)
        c = cls.setdefault(OPCODE_NAMES.get(code, str(code)), {"ms": 0.0, "bytes": 0.0, "macs": 0.0, "ops": 0})
        c["ms"] += t
        c["bytes"] += by * B + wb
        c["macs"] += macs * B
        c["ops"] += 1
    top = max(cls, key=lambda k: cls[k]["ms"])
    peak, peak_src = load_peaks()
    ach = cls[top]["bytes"] / (cls[top]["ms"] / 1e3) / 1e9
    s8_ms = cls.get("pw_s8n", {"ms": 0})["ms"] + cls.get("gemv_s8n", {"ms": 0})["ms"]
    s8_macs = cls.get("pw_s8n", {"macs": 0})["macs"] + cls.get("gemv_s8n", {"macs": 0})["macs"]
    alg_op = cls[top]["bytes"] / cls[top]["ops"]
    traffic, t_ratio, t_what = profile_traffic(top, alg_op)
    roofline = {"bound": "hbm", "kernel": f"{top} ({cls[top]['ops']} ops per step)", "achieved": round(ach, 1),
                "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "traffic": traffic, "traffic_over_algorithmic": t_ratio,
                "algorithmic_bytes_per_op": round(alg_op),
                "peak_source": peak_src,
                "note": "achieved = algorithmic bytes of the op class per step / its CUDA-event time (the per-op "
                        "average); traffic = the class's algorithmic bytes per op x the DRAM / algorithmic ratio of "
                        f"one op captured alone ({t_what}; profiles/traffic_pw_s8n_v24_int8_b64.md)"}
    ops_summary = {k: {"ms": round(v["ms"], 4), "share": round(v["ms"] / sum(x["ms"] for x in cls.values()), 4),
                       "GB/s": round(v["bytes"] / (v["ms"] / 1e3) / 1e9, 1) if v["ms"] else None, "ops": v["ops"]}
                   for k, v in sorted(cls.items(), key=lambda kv: -kv[1]["ms"])}

    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json"), encoding="utf-8") as f:
            bf16 = float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        bf16 = 1590.0  # the profiling recipe's fallback
    c1 = c1_gemm(m, torch, stream, bf16) if rank == 0 else None
    proto = (proto_head_c4(m.h, torch, stream, bf16, cpu=not args.no_cpu_baseline and world == 1)
             if rank == 0 and not args.no_proto else None)
    logmel = (logmel_perch(m.h, torch, stream, load_peaks()[0], cpu=not args.no_cpu_baseline and world == 1)
              if rank == 0 and not args.no_proto else None)
    fp16 = (v24_fp16_c3(torch, stream, cpu=not args.no_cpu_baseline and world == 1)
            if rank == 0 and not args.no_proto else None)
    perch = (perch_c4(torch, stream, cpu=not args.no_cpu_baseline and world == 1)
             if rank == 0 and not args.no_proto else None)
    perch8 = (perch_int8(torch, stream, cpu=not args.no_cpu_baseline and world == 1)
              if rank == 0 and not args.no_proto else None)

    # ---- the library's own split (N > 1): after the ranks' processes are done, rank 0 opens one context over all
    # N GPUs (bnn_set_threads(ctx, N)), scores every rank's windows in one call and compares them with its 1-GPU logits
    single = None
    all_pcm = None
    if world > 1 and rank == 0:
        all_pcm = np.concatenate([synth.audio(B, seed=1000 + r) for r in range(world)])
        ref_out, ref_emb = m.infer_batch(all_pcm)
    launches = m.launches_per_batch
    m.close()
    if world > 1:
        barrier()
        dist.destroy_process_group()
    if world > 1 and rank == 0:
        os.environ["BNN_DEVICES"] = ",".join(str(d) for d in range(world))
        mN = Model(pkg, mode=4, batch=B, devices=world)
        h_all = torch.from_numpy(all_pcm).pin_memory().numpy()
        o_all = torch.empty((world * B, nc), dtype=torch.float32).pin_memory().numpy()
        e_all = torch.empty((world * B, ne), dtype=torch.float32).pin_memory().numpy()
        for _ in range(2):
            mN.infer_batch(h_all, o_all, e_all)
        ts = []
        for _ in range(args.steps):
            t1 = time.perf_counter()
            mN.infer_batch(h_all, o_all, e_all)
            ts.append(time.perf_counter() - t1)
        mN.close()
        sc_ms = float(np.median(ts)) * 1e3
        single = {"value": round(world * B / (sc_ms / 1e3), 3), "unit": UNIT, "gpus": world,
                  "windows_per_call": world * B, "ms_per_call": round(sc_ms, 3),
                  "bit_identical": bool(np.array_equal(o_all.view(np.int32), ref_out.view(np.int32)) and
                                        np.array_equal(e_all.view(np.int32), ref_emb.view(np.int32))),
                  "path": "one context over all GPUs (bnn_set_threads), bnn_infer_batch, pinned host buffers, wall "
                          "clock median; compared with the same windows on one GPU"}

    line = None
    if rank == 0:
        clocks = clk.summary()
        line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8/fp32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "batch_per_gpu": B, "windows_per_step": world * B,
                           "model": "BirdNET-v2.4 architecture, random He-normal weights, 6522-class int8 head",
                           "l2": "inputs larger than L2: 147 MB of PCM per GPU per step (126 MB L2)",
                           "parallelism": f"data parallel over windows, {world} process(es), no collective"},
                "e2e": e2e, "gpu_launches": launches * args.steps, "roofline": roofline,
                "s8_gemm": {"tops": round(2 * s8_macs / (s8_ms / 1e3) / 1e12, 2) if s8_ms else None,
                            "ms_per_step": round(s8_ms, 4),
                            "note": "int8 ops of PW_S8 + GEMV_S8 (quantizer + tcgen05 GEMM) per second; these GEMMs "
                                    "are HBM-bound (AI far below the int8 ridge)"},
                "parity_checked": parity,
                "ops": ops_summary, "clocks": clocks, "s8_gemm_c1": c1, "proto_s8_c4": proto,
                "fe_logmel_perch": logmel, "v24_fp16_c3": fp16, "perch_v2_fp16_s8_c4": perch,
                "perch_v2_int8": perch8,
                "copy_ceiling": copy_ceiling, "bnn_infer_latency": lat}
        if single is not None:
            line["single_context"] = single
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(pkg, pcm)
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
