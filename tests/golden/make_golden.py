"""Generates the golden fixtures of tests/golden from the REFERENCE compiler (run in a checkout that has it).

    python tests/golden/make_golden.py /path/to/birdnet-neon-engine

For each synthetic model (bnneon_b200.synth.v24_ir: the full v2.4 architecture and the 4-block mini variant) the
reference's own lowering (python/bnneon/compiler/lower.py: Lowering, plan_slots) and package writer (pkgfmt.py)
write the neon-int8 package exactly as `bnc.py compile --paths neon-int8 --int8 pw,pwl,head,lin` does after
recognition (cmd_compile.py _lower_path + _set_metadata). The sha256 and size of those packages go into
packages.json; tests/test_package_golden.py checks that bnneon_b200.synth writes byte-identical files, so the loader
and kernels run on the reference compiler's bytes without the reference being present.

It also records the reference packer's output for a few weight matrices (s8_tensors, quant_rows_s8) in
s8_packing.npz.
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


def sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
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


if __name__ == "__main__":
    main()
