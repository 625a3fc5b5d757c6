"""Generates the golden fixtures of tests/golden from the REFERENCE compiler (run in a checkout that has it).

    python tests/golden/make_golden.py /path/to/birdnet-neon-engine

For each synthetic model (bnneon_b200.synth.v24_ir: the full v2.4 architecture and the 4-block mini variant) the
reference's own lowering (python/bnneon/compiler/lower.py: Lowering, plan_slots) and package writer (pkgfmt.py)
write the neon-int8 package exactly as `bnc.py compile --paths neon-int8 --int8 pw,pwl,head,lin` does after
recognition (cmd_compile.py _lower_path + _set_metadata). The sha256 and size of those packages go into
packages.json; tests/test_golden_cpu.py checks that bnneon_b200.synth writes byte-identical files, so the loader
and kernels run on the reference compiler's bytes without the reference being present.

It also records the reference packer's output for a few weight matrices (s8_tensors, quant_rows_s8) in
s8_packing.npz, and for the int8 prototype head (PROTO_S8): the reference lowering's own proto_s8n packs seeded
prototype heads into one-op neon-int8 packages (sha256 in proto_packages.json; bnneon_b200.synth.write_proto_package
must write the same bytes) and its packer (quant_rows_s8, n4_panel_flags, the [Np/4][Kp/16][4][16] layout) runs on
fixed matrices (proto_packing.npz); and the reference lowering's l_fe_logmel writes one-op log-mel front-end packages
(logmel_packages.json), its l_fe_dbimg one-op dB-image front-end packages (dbimg_packages.json) and the Perch-v2-
architecture model on the neon-int8 path with the default int8 policy (perch_int8_packages.json); and the
reference lowering writes the same v2.4 models for the neon-fp16 path (sha256 in
f16_packages.json, with the reference's fp16 SiLU coefficient table read from its source).
"""
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "birdnet-neon-engine_b200"))
from bnneon_b200 import synth  # noqa: E402


def reference_package(ref_root, ir, dst):
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from bnneon.compiler import lower, pkgfmt  # pylint: disable=import-outside-toplevel
    ops, vshape, lv, ev = ir
    pkg = pkgfmt.Package()
    lw = lower.Lowering(pkg, ops, synth.PATH, synth.NSAMP)
    lw.policy["int8"] = synth.INT8_POLICY
    bufs, rops = lw.run(vshape)
    ob, eb = lw.vbuf[lv], lw.vbuf.get(ev)
    n_classes, emb_dim = bufs[ob][3], bufs[eb][3]
    bufs, _ = lower.plan_slots(bufs, rops, [ob, eb])
    pkg.add_path(synth.PATH, lower.path_info(synth.PATH).hwcap, bufs, rops, 0, ob, eb)
    pkg.set(f"src_nodes/{synth.PATH}", "\n".join(lw.src))
    for k, v in synth.metadata(n_classes, emb_dim, synth.labels_for(n_classes)):
        pkg.set(k, v)
    pkg.write(dst)
    return n_classes, emb_dim


# the prototype-head packages the tests use: (name, seed, cells, channels, classes, prototypes per class, ld, eps)
PROTO_HEADS = (("proto_small", 11, 8, 40, 10, 3, 40, 1e-6),
               ("proto_ld", 12, 12, 64, 25, 4, 72, 1e-3),
               ("proto_wide", 13, 300, 96, 9, 2, 96, 1e-6),
               ("proto_mid", 14, 64, 256, 130, 4, 256, 1e-6))


def reference_proto_package(ref_root, head, ld, dst):
    """The reference lowering's PROTO_S8 record (lower.py proto_s8n -> emit_proto) on the input window taken as the
    cells, in a one-op neon-int8 package."""
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from bnneon.compiler import lower, pkgfmt  # pylint: disable=import-outside-toplevel
    n, c = head["P"].shape
    nc, ppc = head["cw"].shape
    ns = head["n_cells"] * ld
    pkg = pkgfmt.Package()
    lw = lower.Lowering(pkg, [], synth.PATH, ns)
    o = {"P": head["P"], "cw": head["cw"], "cb": head["cb"], "eps": head["eps"], "out": "logits"}
    lw.proto_s8n(0, o, 0, head["n_cells"], c, ld, n, nc, ppc)
    ob = lw.vbuf["logits"]
    bufs, _ = lower.plan_slots(lw.bufs, lw.out, [ob])
    pkg.add_path(synth.PATH, lower.path_info(synth.PATH).hwcap, bufs, lw.out, 0, ob, None)
    pkg.set(f"src_nodes/{synth.PATH}", "\n".join(lw.src))
    for k, v in synth.metadata(nc, 0, synth.labels_for(nc), model_id="perch_v2_proto_head_synthetic",
                               family=synth.BNN_MODEL_PERCH_V2, sample_rate=synth.PERCH_SAMPLE_RATE, n_samples=ns,
                               attribution="synthetic prototype head (random weights)"):
        pkg.set(k, v)
    pkg.write(dst)


def proto_fixtures(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from bnneon.compiler import lower, pkgfmt  # pylint: disable=import-outside-toplevel
    out = {}
    with tempfile.TemporaryDirectory() as td:
        for name, seed, p_cells, c, nc, ppc, ld, eps in PROTO_HEADS:
            head = synth.proto_head(seed, p_cells, c, nc, ppc, eps)
            ref = os.path.join(td, name + ".ref.bnpk")
            reference_proto_package(ref_root, head, ld, ref)
            mine = os.path.join(td, name + ".mine.bnpk")
            synth.write_proto_package(mine, head, ld)
            out[name] = dict(seed=seed, cells=p_cells, channels=c, classes=nc, ppc=ppc, ld=ld, eps=eps,
                             size=os.path.getsize(ref), sha256=sha(ref))
            print(name, out[name], "writer matches" if sha(mine) == sha(ref) else "WRITER DIFFERS")
    with open(os.path.join(HERE, "proto_packages.json"), "w", encoding="utf-8") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")
    # the reference packer on fixed matrices: random rows, a zero row, rows that tie at .5, rows whose 32-byte steps
    # overflow an int16 lane of the n=4 loop, and K not a multiple of 32 (no n4 panels)
    rng = np.random.default_rng(21)
    arrays = {}
    mats = [(rng.standard_normal((10, 64)) * 0.5).astype(np.float32),
            (rng.standard_normal((7, 40)) * 2.0).astype(np.float32),
            np.tile(np.array([[2.5, -2.5, 0.5, 1.0] * 16], np.float32), (8, 1)),
            np.concatenate([np.full((4, 96), 1.0, np.float32), (rng.standard_normal((4, 96)) * 0.1).astype(np.float32)]),
            (rng.standard_normal((12, 128)) * 0.3).astype(np.float32)]
    mats[0][3, :] = 0.0
    mats[2][:, 1] = 127.0   # the row maximum: 127 maps to 127 and the rest to (ties) 2.5, 0.5 -> 3, 1
    mats[4][:4, :32] = 40.0  # the first panel: every int16 lane of its first step sums 4 x 127 > 258
    for i, w in enumerate(mats):
        n, c = w.shape
        n_pad, k_pad = (n + 3) & ~3, (c + 15) & ~15
        wq = np.zeros((n_pad, k_pad), np.float32)
        wq[:n, :c] = w
        q, sw = lower.quant_rows_s8(wq)
        arrays[f"w{i}"] = w
        arrays[f"q{i}"] = q
        arrays[f"sw{i}"] = sw
        arrays[f"n4_{i}"] = lower.n4_panel_flags(q)
        arrays[f"qp{i}"] = q.reshape(n_pad // 4, 4, k_pad // 16, 16).transpose(0, 2, 1, 3).copy()
    # the SDOT head's packer (lower.py proto_s8, PROTO variant 2 of the neon-fp16 path) on two of the matrices
    for i in (0, 4):
        w = mats[i]
        n, c = w.shape
        lw = lower.Lowering(pkgfmt.Package(), [], "neon-fp16", 16)
        head = {"P": w, "cw": np.ones((n, 1), np.float32), "cb": np.zeros(n, np.float32), "eps": 1e-6,
                "out": "lg"}
        lw.proto_s8(0, head, 0, 8, c, c, n, n, 1)
        names = [t[0] for t in lw.pkg.tensors]
        arrays[f"sdot_qp{i}"] = lw.pkg.tensors[names.index("s8/proto.0.q")][1]
        arrays[f"sdot_sw{i}"] = lw.pkg.tensors[names.index("s8/proto.0.s")][1]
    np.savez(os.path.join(HERE, "proto_packing.npz"), **arrays)
    print("wrote proto_packages.json and proto_packing.npz")


# the log-mel front-end packages: (name, nsamp, frame, hop, pad, nfft, nmel, floor, scale)
LOGMEL_FES = (("logmel_small", 4000, 400, 160, 0, 512, 40, 1e-5, 1.0),
              ("logmel_odd", 3001, 255, 100, 64, 256, 20, 1e-3, 0.5),
              ("logmel_tiny", 2000, 16, 16, 0, 16, 3, 1e-5, 1.0))


def reference_logmel_package(ref_root, fe, dst):
    """The reference lowering's FE_LOGMEL record (lower.py l_fe_logmel) in a one-op neon-int8 package."""
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from bnneon.compiler import lower, pkgfmt  # pylint: disable=import-outside-toplevel
    pkg = pkgfmt.Package()
    lw = lower.Lowering(pkg, [], synth.PATH, fe["nsamp"])
    o = {"mode": "dft-op", "pad": fe["pad"], "frame": fe["frame"], "hop": fe["hop"], "nfft": fe["nfft"],
         "mel": fe["mel"], "window": fe["window"], "floor": fe["floor"], "scale": fe["scale"], "out": "spec"}
    lw.l_fe_logmel(0, o)
    ob = lw.vbuf["spec"]
    bufs, _ = lower.plan_slots(lw.bufs, lw.out, [ob])
    pkg.add_path(synth.PATH, lower.path_info(synth.PATH).hwcap, bufs, lw.out, 0, ob, None)
    pkg.set(f"src_nodes/{synth.PATH}", "\n".join(lw.src))
    n_out = synth.logmel_frames(fe) * fe["mel"].shape[0]
    for k, v in synth.metadata(n_out, 0, synth.labels_for(n_out), model_id="perch_v2_frontend_synthetic",
                               family=synth.BNN_MODEL_PERCH_V2, sample_rate=synth.PERCH_SAMPLE_RATE,
                               n_samples=fe["nsamp"], attribution="synthetic log-mel front end"):
        pkg.set(k, v)
    pkg.write(dst)


def logmel_fixtures(ref_root):
    out = {}
    with tempfile.TemporaryDirectory() as td:
        for name, nsamp, frame, hop, pad, nfft, nmel, floor, scale in LOGMEL_FES:
            fe = synth.logmel_frontend(nsamp, frame, hop, pad, nfft, nmel, floor=floor, scale=scale)
            ref = os.path.join(td, name + ".ref.bnpk")
            reference_logmel_package(ref_root, fe, ref)
            mine = os.path.join(td, name + ".mine.bnpk")
            synth.write_logmel_package(mine, fe)
            out[name] = dict(nsamp=nsamp, frame=frame, hop=hop, pad=pad, nfft=nfft, nmel=nmel, floor=floor,
                             scale=scale, size=os.path.getsize(ref), sha256=sha(ref))
            print(name, out[name], "writer matches" if sha(mine) == sha(ref) else "WRITER DIFFERS")
    with open(os.path.join(HERE, "logmel_packages.json"), "w", encoding="utf-8") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")


# the neon-fp16 packages: (name, seed, blocks, head classes); 61 classes give the fp32 head (DENSE variant 0)
F16_MODELS = (("v24_full_f16", 0, "full", 6522), ("v24_mini_f16", 1, "mini", 100), ("v24_mini_f16_h32", 1, "mini", 61))


def reference_f16_package(ref_root, ir, dst):
    """The reference lowering of the v2.4 IR for the neon-fp16 path (bnc.py compile --paths neon-fp16)."""
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from bnneon.compiler import lower, pkgfmt  # pylint: disable=import-outside-toplevel
    ops, vshape, lv, ev = ir
    pkg = pkgfmt.Package()
    lw = lower.Lowering(pkg, ops, synth.PATH_F16, synth.NSAMP)
    bufs, rops = lw.run(vshape)
    ob, eb = lw.vbuf[lv], lw.vbuf.get(ev)
    n_classes, emb_dim = bufs[ob][3], bufs[eb][3]
    bufs, _ = lower.plan_slots(bufs, rops, [ob, eb])
    pkg.add_path(synth.PATH_F16, lower.path_info(synth.PATH_F16).hwcap, bufs, rops, 0, ob, eb)
    pkg.set(f"src_nodes/{synth.PATH_F16}", "\n".join(lw.src))
    for k, v in synth.metadata(n_classes, emb_dim, synth.labels_for(n_classes)):
        pkg.set(k, v)
    pkg.write(dst)
    return n_classes, emb_dim


def silu_table(ref_root):
    """The fp16 SiLU table of the reference (src/silu_lut_tables_deg2.h: low bytes then high bytes of 16 fp16
    coefficients per array) as 16-bit values."""
    import re  # pylint: disable=import-outside-toplevel
    with open(os.path.join(ref_root, "src", "silu_lut_tables_deg2.h"), encoding="utf-8") as f:
        text = f.read()
    out = {}
    for name in ("C0", "C1", "C2"):
        body = re.search(r"SILU_LUT_%s\[32\][^{]*\{([^}]*)\}" % name, text).group(1)
        b = [int(x, 16) for x in re.findall(r"0x[0-9a-fA-F]+", body)]
        out[name.lower()] = [b[i] | b[16 + i] << 8 for i in range(16)]
    return out


def f16_fixtures(ref_root):
    out = {}
    with tempfile.TemporaryDirectory() as td:
        for name, seed, kind, nc in F16_MODELS:
            blocks = synth.V24_BLOCKS if kind == "full" else synth.MINI_BLOCKS
            ref = os.path.join(td, name + ".ref.bnpk")
            n_classes, emb_dim = reference_f16_package(ref_root, synth.v24_ir(seed, nc, blocks), ref)
            mine = os.path.join(td, name + ".mine.bnpk")
            synth.write_f16_package(mine, synth.v24_ir(seed, nc, blocks))
            out[name] = dict(seed=seed, blocks=kind, head_classes=nc, n_classes=n_classes, emb_dim=emb_dim,
                             size=os.path.getsize(ref), sha256=sha(ref))
            print(name, out[name], "writer matches" if sha(mine) == sha(ref) else "WRITER DIFFERS")
    out["silu_lut"] = silu_table(ref_root)
    with open(os.path.join(HERE, "f16_packages.json"), "w", encoding="utf-8") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")


# the one-op dB-image front-end packages (FE_DBIMG): keyword arguments of synth.dbimg_frontend (chan None: the seeded
# mean / std pair)
DBIMG_FES = {
    "dbimg_v3": dict(synth.V3_FE, rows=list(synth.V3_FE["rows"])),
    "dbimg_small": dict(nsamp=8000, nfft=256, hop=100, pad=128, pad_mode="reflect", nmel=40, rows=list(range(32)),
                        Ho=48, Wo=64, C=3, top_db=80.0, norm=1),
    "dbimg_zero": dict(nsamp=6000, nfft=512, hop=256, pad=256, pad_mode="zero", nmel=64, rows=list(range(50, 10, -1)),
                       Ho=20, Wo=30, C=5, top_db=None, norm=2, post=[[1, 4.3429448], [3, -5.0], [2, 2.0]],
                       chan=[[1, [0.5, 1.0, 1.5, 2.0, 2.5]], [3, [0.0, -0.25, 0.25, 1.0, -1.0]]]),
    "dbimg_none": dict(nsamp=4096, nfft=64, hop=64, pad=0, pad_mode="none", nmel=8, rows=[7, 0, 3], Ho=3, Wo=64, C=1,
                       top_db=10.0, norm=0, post=[], chan=[]),
}


def dbimg_frontend(g):
    g = dict(g)
    if g.get("post") is not None:
        g["post"] = [(int(c), float(v)) for c, v in g["post"]]
    if g.get("chan") is not None:
        g["chan"] = [(int(c), np.asarray(v, np.float32)) for c, v in g["chan"]]
    return synth.dbimg_frontend(**g)


def reference_dbimg_package(ref_root, fe, dst):
    """The reference lowering's FE_DBIMG record (lower.py l_fe_dbimg) in a one-op neon-int8 package."""
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from bnneon.compiler import lower, pkgfmt  # pylint: disable=import-outside-toplevel
    pkg = pkgfmt.Package()
    lw = lower.Lowering(pkg, [], synth.PATH, fe["nsamp"])
    o = dict(fe, out="img")
    lw.l_fe_dbimg(0, o)
    ob = lw.vbuf["img"]
    bufs, _ = lower.plan_slots(lw.bufs, lw.out, [ob])
    pkg.add_path(synth.PATH, lower.path_info(synth.PATH).hwcap, bufs, lw.out, 0, ob, None)
    pkg.set(f"src_nodes/{synth.PATH}", "\n".join(lw.src))
    ld = fe["C"] if fe["C"] % 4 == 0 else (fe["C"] + 3) & ~3
    n_out = fe["Ho"] * fe["Wo"] * ld
    for k, v in synth.metadata(n_out, 0, synth.labels_for(n_out), model_id="birdnet_v3_frontend_synthetic",
                               family=synth.BNN_MODEL_BIRDNET_V3, sample_rate=synth.V3_SAMPLE_RATE,
                               n_samples=fe["nsamp"], attribution="synthetic dB-image front end"):
        pkg.set(k, v)
    pkg.write(dst)


def dbimg_fixtures(ref_root):
    out = {}
    with tempfile.TemporaryDirectory() as td:
        for name, g in DBIMG_FES.items():
            fe = dbimg_frontend(g)
            ref = os.path.join(td, name + ".ref.bnpk")
            reference_dbimg_package(ref_root, fe, ref)
            mine = os.path.join(td, name + ".mine.bnpk")
            synth.write_dbimg_package(mine, fe)
            out[name] = dict(frontend=g, size=os.path.getsize(ref), sha256=sha(ref))
            print(name, out[name]["size"], "writer matches" if sha(mine) == sha(ref) else "WRITER DIFFERS")
    with open(os.path.join(HERE, "dbimg_packages.json"), "w", encoding="utf-8") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")


def perch_ir_for_reference(ops):
    """perch_ir()'s ops with the log-mel front end in the reference lowering's own node form (l_fe_logmel)"""
    out = []
    for o in ops:
        o = dict(o)
        if o["op"] == "FE_LOGMEL":
            fe = o.pop("fe")
            o.update(mode="dft-op", pad=fe["pad"], frame=fe["frame"], hop=fe["hop"], nfft=fe["nfft"], mel=fe["mel"],
                     window=fe["window"], floor=fe["floor"], scale=fe["scale"])
        out.append(o)
    return out


def reference_perch_int8_package(ref_root, ir, dst):
    """The reference lowering of the Perch-v2-architecture IR for the neon-int8 path with its default int8 policy
    (bnc.py compile --paths neon-int8)."""
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from bnneon.compiler import lower, pkgfmt  # pylint: disable=import-outside-toplevel
    ops, vshape, lv, ev, fe = ir
    pkg = pkgfmt.Package()
    lw = lower.Lowering(pkg, perch_ir_for_reference(ops), synth.PATH, fe["nsamp"])
    bufs, rops = lw.run(vshape)
    ob, eb = lw.vbuf[lv], lw.vbuf[ev]
    n_classes, emb_dim = bufs[ob][3], bufs[eb][3]
    bufs, _ = lower.plan_slots(bufs, rops, [ob, eb])
    pkg.add_path(synth.PATH, lower.path_info(synth.PATH).hwcap, bufs, rops, 0, ob, eb)
    pkg.set(f"src_nodes/{synth.PATH}", "\n".join(lw.src))
    for k, v in synth.metadata(n_classes, emb_dim, synth.labels_for(n_classes), model_id="perch_v2_synthetic",
                               family=synth.BNN_MODEL_PERCH_V2, sample_rate=synth.PERCH_SAMPLE_RATE,
                               n_samples=fe["nsamp"],
                               attribution="synthetic Perch-v2-architecture model (random weights)"):
        pkg.set(k, v)
    pkg.write(dst)
    return n_classes, emb_dim


def perch_int8_fixtures(ref_root):
    out = {}
    with tempfile.TemporaryDirectory() as td:
        for name, mini in (("perch_v2_int8_mini", True), ("perch_v2_int8", False)):
            ref = os.path.join(td, name + ".ref.bnpk")
            n_classes, emb_dim = reference_perch_int8_package(ref_root, synth.perch_ir(0, mini=mini), ref)
            mine = os.path.join(td, name + ".mine.bnpk")
            synth.write_perch_int8_package(mine, synth.perch_ir(0, mini=mini))
            out[name] = dict(seed=0, mini=mini, n_classes=n_classes, emb_dim=emb_dim, size=os.path.getsize(ref),
                             sha256=sha(ref))
            print(name, out[name], "writer matches" if sha(mine) == sha(ref) else "WRITER DIFFERS")
    with open(os.path.join(HERE, "perch_int8_packages.json"), "w", encoding="utf-8") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")


def sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <checkout of the reference repository>")
    ref_root = sys.argv[1]
    out = {}
    with tempfile.TemporaryDirectory() as td:
        for name, seed, blocks, nc in (("v24_full", 0, synth.V24_BLOCKS, 6522),
                                       ("v24_mini", 1, synth.MINI_BLOCKS, 61)):
            ir = synth.v24_ir(seed, nc, blocks)
            ref = os.path.join(td, name + ".ref.bnpk")
            n_classes, emb_dim = reference_package(ref_root, ir, ref)
            mine = os.path.join(td, name + ".mine.bnpk")
            synth.write_int8_package(mine, synth.v24_ir(seed, nc, blocks))
            out[name] = dict(seed=seed, head_classes=nc, n_classes=n_classes, emb_dim=emb_dim,
                             size=os.path.getsize(ref), sha256=sha(ref))
            print(name, out[name], "writer matches" if sha(mine) == sha(ref) else "WRITER DIFFERS")
    with open(os.path.join(HERE, "packages.json"), "w", encoding="utf-8") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")

    # the reference packer on fixed matrices
    sys.path.insert(0, os.path.join(ref_root, "python"))
    from bnneon.compiler import lower, pkgfmt  # pylint: disable=import-outside-toplevel
    rng = np.random.default_rng(7)
    arrays = {}
    for i, (n, k) in enumerate(((5, 3), (24, 48), (36, 72), (13, 100))):
        w = (rng.standard_normal((n, k)) * 0.3).astype(np.float32)
        w[0, :] = 0.0
        b = rng.standard_normal(n).astype(np.float32)
        lw = lower.Lowering(pkgfmt.Package(), [], synth.PATH, 16)
        tl, shp = lw.s8_tensors("t", w, b)
        arrays[f"w{i}"] = w
        arrays[f"bias{i}"] = b
        arrays[f"shape{i}"] = np.array(shp, np.int32)
        for j, suffix in enumerate(("q", "sw", "cs", "b")):
            arrays[f"{suffix}{i}"] = lw.pkg.tensors[tl[j]][1]
    np.savez(os.path.join(HERE, "s8_packing.npz"), **arrays)
    print("wrote packages.json and s8_packing.npz")
    proto_fixtures(ref_root)
    logmel_fixtures(ref_root)
    f16_fixtures(ref_root)
    dbimg_fixtures(ref_root)
    perch_int8_fixtures(ref_root)


if __name__ == "__main__":
    main()
