"""Synthetic BirdNET-v2.4-architecture models and audio, and a writer for their neon-int8 packages.

There is no BirdNET v2.4 ONNX file here (and no network), so the benchmark and the tests run a model of the v2.4
architecture with seeded random weights:

* ``v24_ir(seed)`` builds the fused intermediate representation the reference compiler lowers (the op dicts of
  python/bnneon/compiler/recog.py after fusion: FE_STFT2_POW, CONV, DWCONV, SE, AFFINE, MEAN, DENSE) with the layer
  shapes of results/graph_compact.txt and results/mac_table.txt: front end 2048/278 + 1024/280 on 144000 samples,
  c0 4x8 stride 2 + ReLU + max|avg pool, p0 1x1, 16 inverted-residual blocks (b1.1-b4.4, SE on b2-b4), post BN +
  ReLU + 3x3 pc conv + mean (the 1024-d embedding), and a dense head.
* ``write_int8_package(path, ir)`` writes the ``neon-int8`` package the reference compiler would write for that IR
  with the int8 policy ``pw,pwl,head,lin`` (bnc.py compile --paths neon-int8 --int8 pw,pwl,head,lin). The output is
  byte-identical to the reference compiler's (the sha256 is pinned in tests/golden/packages.json, produced by
  tests/golden/make_golden.py with the reference's own lower.py / pkgfmt.py), so the loader and the kernels are
  tested on genuine package bytes.
* ``audio(n, seed)`` makes seeded windows of noise plus linear chirps.

Weights: He-normal N(0, sqrt(2 / fan_in)) for every expanding conv and the dense layers; the projecting 1x1 convs
(pwl) use half of the LeCun scale so that the residual stack stays in range without batch norm; biases are small
seeded normals. The front end uses periodic Hann windows and triangular mel filter banks below Nyquist.
"""
import hashlib
import struct

import numpy as np

NSAMP = 144000
SAMPLE_RATE = 48000

# (tag, stride, c_in, c_mid, c_out, se_rd, residual): results/mac_table.txt:3-53, results/graph_compact.txt
V24_BLOCKS = (
    [("b1.1", 2, 24, 72, 36, 0, False), ("b1.2", 1, 36, 72, 36, 0, True), ("b1.3", 1, 36, 72, 36, 0, True),
     ("b2.1", 2, 36, 288, 72, 18, False)]
    + [(f"b2.{i}", 1, 72, 288, 72, 18, True) for i in (2, 3, 4)]
    + [("b3.1", 2, 72, 864, 108, 27, False)]
    + [(f"b3.{i}", 1, 108, 864, 108, 27, True) for i in (2, 3, 4, 5)]
    + [("b4.1", 2, 108, 1536, 192, 48, False)]
    + [(f"b4.{i}", 1, 192, 1536, 192, 48, True) for i in (2, 3, 4)])
# the same stages with one (strided) block each: the same op kinds and end geometry, for quick tests
MINI_BLOCKS = tuple(b for b in V24_BLOCKS if b[0].endswith(".1"))

INT8_POLICY = "pw,pwl,head,lin"
PATH = "neon-int8"


# ------------------------------------------------------------------ the model IR

def _mel_bank(nfft, fmin, fmax, nmel=96, rate=None):
    """Triangular filters on the HTK mel scale, [nmel][nfft/2 + 1] float32, zero at and above fmax."""
    bins = nfft // 2 + 1
    mel = lambda f: 2595.0 * np.log10(1.0 + f / 700.0)  # noqa: E731
    imel = lambda m: 700.0 * (10.0 ** (m / 2595.0) - 1.0)  # noqa: E731
    edges = imel(np.linspace(mel(fmin), mel(fmax), nmel + 2))
    freqs = np.arange(bins) * (rate or SAMPLE_RATE) / nfft
    out = np.zeros((nmel, bins), np.float64)
    for j in range(nmel):
        lo, c, hi = edges[j], edges[j + 1], edges[j + 2]
        up = (freqs - lo) / max(c - lo, 1e-9)
        down = (hi - freqs) / max(hi - c, 1e-9)
        out[j] = np.maximum(0.0, np.minimum(up, down))
    return out.astype(np.float32)


def _hann(n):
    return (0.5 - 0.5 * np.cos(2 * np.pi * np.arange(n) / n)).astype(np.float32)


def v24_ir(seed=0, n_classes=6522, blocks=V24_BLOCKS):
    """The fused IR of a v2.4-architecture model with seeded random weights.

    Returns:
        (ops, vshape, logits_value, embedding_value): ops as the reference compiler's recognizer emits them after
        fusion, vshape {value id: (H, W)}.
    """
    rng = np.random.default_rng(seed)
    f32 = np.float32

    def he(*shape, fan_in, scale=1.0):
        return (rng.standard_normal(shape) * (scale * np.sqrt(2.0 / fan_in))).astype(f32)

    def bias(n, s=0.02):
        return (rng.standard_normal(n) * s).astype(f32)

    ops, vshape = [], {}
    nid = [0]

    def val(h, w):
        nid[0] += 1
        vshape[nid[0]] = (h, w)
        return nid[0]

    img = val(96, 511)
    ops.append(dict(op="FE_STFT2_POW", ins=[], out=img, eps=1e-6,
                    branches=[dict(nfft=2048, hop=278, window=_hann(2048), dft=None,
                                   mel=_mel_bank(2048, 0.0, 3000.0), pow=0.25),
                              dict(nfft=1024, hop=280, window=_hann(1024), dft=None,
                                   mel=_mel_bank(1024, 500.0, 15000.0), pow=0.3)],
                    bn_s=np.array([0.8, 1.1], f32), bn_b=np.array([-0.2, 0.1], f32),
                    nodes=["v24/fe"]))
    c0 = val(48, 128)
    ops.append(dict(op="CONV", ins=[img], out=c0, w=he(24, 2, 4, 8, fan_in=64), b=bias(24), k=[4, 8], s=[2, 2],
                    pads=[1, 3, 1, 4], act="relu", pool="maxavg_w2", nodes=["v24/c0"]))
    x = val(48, 128)
    ops.append(dict(op="CONV", ins=[c0], out=x, w=he(24, 48, 1, 1, fan_in=48), b=bias(24), k=[1, 1], s=[1, 1],
                    pads=[0, 0, 0, 0], act=None, nodes=["v24/p0"]))
    h, w = 48, 128
    for tag, st, cin, cm, cout, rd, skip in blocks:
        ho, wo = (h + 2 - 3) // st + 1, (w + 2 - 3) // st + 1
        e = val(h, w)
        ops.append(dict(op="CONV", ins=[x], out=e, w=he(cm, cin, 1, 1, fan_in=cin), b=bias(cm), k=[1, 1], s=[1, 1],
                        pads=[0, 0, 0, 0], act="swish", nodes=[f"v24/{tag}/pw"]))
        d = val(ho, wo)
        ops.append(dict(op="DWCONV", ins=[e], out=d, w=he(cm, 1, 3, 3, fan_in=9), b=bias(cm), k=[3, 3],
                        s=[st, st], pads=[1, 1, 1, 1], act="swish", nodes=[f"v24/{tag}/dw"]))
        if rd:
            g = val(ho, wo)
            ops.append(dict(op="SE", ins=[d], out=g, w1=he(rd, cm, fan_in=cm), b1=bias(rd), act1="swish",
                            w2=he(cm, rd, fan_in=rd), b2=bias(cm, 0.5), nodes=[f"v24/{tag}/se"]))
            d = g
        y = val(ho, wo)
        pwl = dict(op="CONV", ins=[d], out=y, w=he(cout, cm, 1, 1, fan_in=cm, scale=0.35), b=bias(cout), k=[1, 1],
                   s=[1, 1], pads=[0, 0, 0, 0], act=None, nodes=[f"v24/{tag}/pwl"])
        if skip:
            pwl["res"] = x
        ops.append(pwl)
        x, h, w = y, ho, wo
    a = val(h, w)
    ops.append(dict(op="AFFINE", ins=[x], out=a, s=(1.0 + 0.1 * rng.standard_normal(192)).astype(f32),
                    t=bias(192, 0.1), act="relu", nodes=["v24/post_bn"]))
    pc = val(1, 6)
    ops.append(dict(op="CONV", ins=[a], out=pc, w=he(1024, 192, 3, 3, fan_in=1728), b=bias(1024), k=[3, 3],
                    s=[1, 1], pads=[0, 0, 0, 0], act="relu", nodes=["v24/pc"]))
    feat = val(1, 1)
    ops.append(dict(op="MEAN", ins=[pc], out=feat, nodes=["v24/mean"]))
    logits = val(1, 1)
    ops.append(dict(op="DENSE", ins=[feat], out=logits, w=he(n_classes, 1024, fan_in=1024, scale=0.5),
                    b=bias(n_classes), nodes=["v24/head"]))
    return ops, vshape, logits, feat


def labels_for(n_classes):
    """A label file (bytes) with one synthetic class name per line."""
    return "".join(f"Synthetic species {i:05d}_Synthetic {i:05d}\n" for i in range(n_classes)).encode()


def metadata(n_classes, emb_dim, labels, model_id="birdnet_v2.4_synthetic", family=24, sample_rate=SAMPLE_RATE,
             n_samples=NSAMP, attribution="synthetic BirdNET-v2.4-architecture model (random weights)"):
    """The package metadata records, in the compiler's order (cmd_compile.py _set_metadata)."""
    return [("model_id", model_id), ("family", family), ("sample_rate", sample_rate), ("n_samples", n_samples),
            ("hop_samples", 0), ("n_classes", int(n_classes)), ("emb_dim", int(emb_dim)), ("post", 1),
            ("logit_scale", 1.0), ("labels_sha256", hashlib.sha256(labels).digest()), ("labels_file", "labels.txt"),
            ("labels", labels), ("license", "synthetic weights, no license restrictions"),
            ("attribution", attribution),
            ("source_sha256", "0" * 64),
            ("input", f"float32 PCM in [-1, 1) at sample_rate, {n_samples} samples per window"),
            ("compiler", "bnc 3")]


# ------------------------------------------------------------------ the neon-int8 lowering of that IR

F32, F16, I8, I32 = 0, 1, 2, 3
OPC = dict(FE_STFT2=1, C0POOL=2, DW3=4, POSTPC=6, PW_S8=22, GEMV_S8=23, SE_GATE=25)
OPC_PW_F32 = 3


def _r8(x):
    return (x + 7) & ~7


def _r16(x):
    return (x + 15) & ~15


class _Int8Lowering:
    """The neon-int8 lowering of the v2.4 IR (pw, pwl, head and dense layers on int8).

    Follows the reference compiler's rules for these op kinds (python/bnneon/compiler/lower.py: buffer shapes and
    element counts, tensor names and packing, op records and their int parameters, the order buffers and tensors are
    created in), so the package it produces is the reference compiler's.
    """

    def __init__(self, ops):
        self.ops = ops
        self.bufs = [(F32, 1, 1, NSAMP, NSAMP, 0, NSAMP)]
        self.tensors, self.tindex = [], {}
        self.records, self.src = [], []
        self.vbuf, self.gate, self.uses = {}, {}, {}
        self.chsum = (None, None)
        for o in ops:
            for i in o["ins"] + ([o["res"]] if o.get("res") else []):
                self.uses.setdefault(i, []).append(o)

    # helpers
    def buf(self, dt, h, w, c, ld=None, halo=0, elems=None):
        ld = ld or c
        if elems is None:
            elems = (h + 2 * halo) * (w + 2 * halo) * ld if halo else _r8(h * w) * ld
        self.bufs.append((dt, h, w, c, ld, halo, int(elems)))
        return len(self.bufs) - 1

    def tensor(self, name, a):
        if name in self.tindex:
            return self.tindex[name]
        a = np.ascontiguousarray(a)
        self.tindex[name] = len(self.tensors)
        self.tensors.append((name, a))
        return self.tindex[name]

    def emit(self, code, bl, tl, il, o):
        self.records.append((code, [int(x) for x in bl], [int(x) for x in tl], [int(x) for x in il]))
        n = [x for x in o.get("nodes", []) if x] or ["?"]
        self.src.append(f"'{n[0]}'" + (f" +{len(n) - 1}" if len(n) > 1 else "") if o.get("nodes") else "?")

    @staticmethod
    def pack_f32(w, b, kp):
        n, k = w.shape
        np_ = _r8(n)
        panels = np.zeros((((np_ * kp * 4) + 127) & ~63) // 4, np.float32)
        w32 = np.zeros((np_, k), np.float32)
        w32[:n] = w
        panels[:np_ * kp].reshape(np_ // 8, kp, 8)[:, :k, :] = w32.reshape(np_ // 8, 8, k).transpose(0, 2, 1)
        bb = np.zeros(np_ + 8, np.float32)
        bb[:n] = b
        return panels, bb, (n, k, kp, np_)

    def s8(self, tag, w, b):
        """per-output-channel symmetric int8, ties away from zero, panels [Np/4][Kp/16][4][16] (lower.py:883-914)"""
        n, k = w.shape
        np_, kp = _r8(n), _r16(k)
        wq = np.zeros((np_, kp), np.float64)
        wq[:n, :k] = w
        am = np.abs(wq).max(1)
        sw = np.where(am > 0, am / 127.0, 1.0)
        ws = wq / sw[:, None]
        q = np.clip(np.sign(ws) * np.floor(np.abs(ws) + 0.5), -127, 127).astype(np.int8)
        panels = q.reshape(np_ // 4, 4, kp // 16, 16).transpose(0, 2, 1, 3).copy()
        cs = q.astype(np.int32).sum(1).astype(np.int32)
        bb = np.zeros(np_ + 8, np.float32)
        bb[:n] = b
        swf = np.zeros(np_ + 8, np.float32)
        swf[:np_] = sw
        csp = np.zeros(np_ + 8, np.int32)
        csp[:np_] = cs
        t = [self.tensor(f"s8n/{tag}.q", panels), self.tensor(f"s8n/{tag}.sw", swf),
             self.tensor(f"s8n/{tag}.cs", csp), self.tensor(f"s8n/{tag}.b", bb)]
        return t, (n, k, kp, np_)

    def out_buffer(self, o, ho, wo, co):
        cons = self.uses.get(o["out"], [])
        if len(cons) == 1 and cons[0]["op"] == "DWCONV" and co % 8 == 0:
            return self.buf(F32, ho, wo, co, ld=co, halo=1), wo, 1, co
        ldo = _r8(co)
        return self.buf(F32, ho, wo, co, ld=ldo), 0, 0, ldo

    # op kinds
    def run(self):
        i = 0
        k = 0
        while i < len(self.ops):
            o = self.ops[i]
            i = getattr(self, "l_" + o["op"].lower())(i, o, k)
            k += 1

    def l_fe_stft2_pow(self, i, o, k):
        b1, b2 = o["branches"]
        tl = [self.tensor("fe/win1", b1["window"]), self.tensor("fe/win2", b2["window"]),
              self.tensor("fe/mel1", b1["mel"]), self.tensor("fe/mel2", b2["mel"]),
              self.tensor("fe/pow1", np.array([b1["pow"]], np.float32)),
              self.tensor("fe/pow2", np.array([b2["pow"]], np.float32)),
              self.tensor("fe/bn_s", o["bn_s"]), self.tensor("fe/bn_b", o["bn_b"])]
        ob = self.buf(F32, 96, 511, 2)
        self.emit(OPC["FE_STFT2"], [0, ob], tl, [], o)
        self.vbuf[o["out"]] = ob
        return i + 1

    def l_conv(self, i, o, k):
        w, b = o["w"], o["b"]
        co = w.shape[0]
        ib = self.vbuf[o["ins"][0]]
        if o["k"] == [4, 8]:  # c0 + ReLU + max|avg pool
            panels, bb, shp = self.pack_f32(w.transpose(0, 2, 3, 1).reshape(co, -1), b, 64)
            tl = [self.tensor(f"s8n/c0.{k}.w", panels), self.tensor(f"s8n/c0.{k}.b", bb)]
            ob = self.buf(F32, 48, 128, 48)
            self.emit(OPC["C0POOL"], [ib, ob], tl, list(shp), o)
            self.vbuf[o["out"]] = ob
            return i + 1
        _, h_in, w_in, _, ld, _, _ = self.bufs[ib]
        tl, shp = self.s8(f"pw.{k}", w[:, :, 0, 0], b)
        ob, ow, opad, ldo = self.out_buffer(o, h_in, w_in, co)
        rb, ldr = -1, 0
        if o.get("res"):
            rb = self.vbuf[o["res"]]
            ldr = self.bufs[rb][4]
        gate = [self.gate[o["ins"][0]]] if o["ins"][0] in self.gate else []
        m4 = (h_in * w_in + 3) & ~3
        qb = self.buf(I8, m4, 1, shp[2])
        sb = self.buf(F32, m4, 1, 1)
        zb = self.buf(I32, m4, 1, 1)
        act = {None: 0, "swish": 1, "relu": 2}[o.get("act")]
        self.emit(OPC["PW_S8"], [ib, ob, rb, qb, sb, zb] + gate, tl,
                  list(shp) + [h_in * w_in, ld, act, ldo, ow, opad, ldr], o)
        self.vbuf[o["out"]] = ob
        return i + 1

    def l_dwconv(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        _, h, w, c, _, _, _ = self.bufs[ib]
        ho, wo = self.vshape[o["out"]]
        self.bufs.append((F32, 1, 1, c, c, 0, c))
        cs = len(self.bufs) - 1
        ob = self.buf(F32, ho, wo, c)
        w9 = o["w"][:, 0].transpose(1, 2, 0).reshape(9, c)
        tl = [self.tensor(f"s8n/dw.{k}.w", w9.astype(np.float32)),
              self.tensor(f"s8n/dw.{k}.b", o["b"].astype(np.float32))]
        self.emit(OPC["DW3"], [ib, ob, cs], tl, [h, w, c, o["s"][0], ho, wo], o)
        self.vbuf[o["out"]] = ob
        self.chsum = (ob, cs)
        return i + 1

    def l_se(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        cs = self.chsum[1]
        _, h, w, c, _, _, _ = self.bufs[ib]
        rd = o["w1"].shape[0]
        tl = [self.tensor(f"s8n/se.{k}.w1", o["w1"]), self.tensor(f"s8n/se.{k}.b1", o["b1"]),
              self.tensor(f"s8n/se.{k}.w2t", np.ascontiguousarray(o["w2"].T)),
              self.tensor(f"s8n/se.{k}.b2", o["b2"])]
        gb = self.buf(F32, 1, 1, c, elems=c)
        self.emit(OPC["SE_GATE"], [cs, gb], tl, [c, rd, h * w], o)
        self.gate[o["out"]] = gb
        self.vbuf[o["out"]] = ib
        return i + 1

    def l_affine(self, i, o, k):
        nx, mn = self.ops[i + 1], self.ops[i + 2]
        ib = self.vbuf[o["ins"][0]]
        w = nx["w"].transpose(0, 2, 3, 1).reshape(1024, 1728)
        panels, bb, shp = self.pack_f32(w, nx["b"], 1728)
        tl = [self.tensor(f"s8n/pc.{k}.w", panels), self.tensor(f"s8n/pc.{k}.b", bb)]
        tl = [self.tensor(f"s8n/post.{k}.s", o["s"]), self.tensor(f"s8n/post.{k}.t", o["t"])] + tl
        fb = self.buf(F32, 1, 1, 1024)
        pin = self.buf(F32, 8, 1, 1728)
        pout = self.buf(F32, 8, 1, 1024)
        self.emit(OPC["POSTPC"], [ib, fb, pin, pout], tl, list(shp), o)
        self.vbuf[mn["out"]] = fb
        return i + 3

    def l_dense(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        n = o["w"].shape[0]
        self.buf(F32, 1, 1, n)  # the compiler allocates the fp32 head's output before choosing the int8 head
        tl, shp = self.s8(f"gemv.{k}", o["w"], o["b"])
        ob = self.buf(F32, 1, 1, shp[3])
        qb = self.buf(I8, 4, 1, shp[2])
        sb = self.buf(F32, 4, 1, 1)
        zb = self.buf(I32, 4, 1, 1)
        self.emit(OPC["GEMV_S8"], [ib, ob, qb, sb, zb], tl, list(shp) + [0], o)
        self.vbuf[o["out"]] = ob
        return i + 1


OPC_F16 = dict(C0POOL=0x102, PW=0x103, DW3=0x104, SE=0x105, POSTPC=0x106, DENSE=0x107)
OPC_DENSE_F32 = 7
PATH_F16 = "neon-fp16"


def pack_h16(w, b, kp):
    """hp_pack (src/gemm_f16.c:17-40, lower.py pack_h16): fp16 panels [Np/16][Kp][16] and, when Np % 16, a [Kp][8] tail
    panel; the bias as fp32 and as fp16, [Np + 16] each."""
    n, k = w.shape
    np_ = _r8(n)
    n16 = np_ // 16
    panels = np.zeros((((np_ * kp * 2) + 127) & ~63) // 2, np.float16)
    w16 = np.zeros((np_, k), np.float16)
    w16[:n] = w
    panels[:n16 * kp * 16].reshape(n16, kp, 16)[:, :k, :] = w16[:n16 * 16].reshape(n16, 16, k).transpose(0, 2, 1)
    if np_ > n16 * 16:
        at = n16 * kp * 16
        panels[at:at + kp * 8].reshape(kp, 8)[:k, :] = w16[n16 * 16:].T
    b32 = np.zeros(np_ + 16, np.float32)
    b32[:n] = b
    return panels, b32, b32.astype(np.float16), (n, k, kp, np_)


class _F16Lowering(_Int8Lowering):
    """The neon-fp16 lowering of the v2.4 IR: fp16 activations, fp16 GEMM panels (hp_pack), fp16 depthwise weights,
    the SE applied in place, the fp16 post conv and an fp16 head (fp32 for heads of 64 classes or fewer).

    Follows python/bnneon/compiler/lower.py for the "neon-fp16" path (PathInfo act fp16, variant 1, prefix "f16/";
    l_conv, pw, out_for_dw, l_dwconv, l_se, l_affine, l_dense), so the package it writes is the reference compiler's.
    """

    def gemm_tensors(self, tag, w, b, kp):
        panels, b32, b16, shp = pack_h16(w, b, kp)
        return [self.tensor(f"f16/{tag}.w", panels), self.tensor(f"f16/{tag}.b32", b32),
                self.tensor(f"f16/{tag}.b16", b16)], shp

    def l_conv(self, i, o, k):
        w, b = o["w"], o["b"]
        co = w.shape[0]
        ib = self.vbuf[o["ins"][0]]
        if o["k"] == [4, 8]:  # c0 + ReLU + max|avg pool
            tl, shp = self.gemm_tensors(f"c0.{k}", w.transpose(0, 2, 3, 1).reshape(co, -1), b, 64)
            ob = self.buf(F16, 48, 128, 48)
            self.emit(OPC_F16["C0POOL"], [ib, ob], tl, list(shp), o)
            self.vbuf[o["out"]] = ob
            return i + 1
        _, h_in, w_in, _, ld, _, _ = self.bufs[ib]
        tl, shp = self.gemm_tensors(f"pw.{k}", w[:, :, 0, 0], b, _r8(w.shape[1]))
        cons = self.uses.get(o["out"], [])
        if len(cons) == 1 and cons[0]["op"] == "DWCONV" and co % 8 == 0:
            ob, ow, opad, ldo = self.buf(F16, h_in, w_in, co, ld=co, halo=1), w_in, 1, co
        else:
            ldo = _r8(co)
            ob, ow, opad = self.buf(F16, h_in, w_in, co, ld=ldo), 0, 0
        rb, ldr = -1, 0
        if o.get("res"):
            rb = self.vbuf[o["res"]]
            ldr = self.bufs[rb][4]
        act = {None: 0, "swish": 1, "relu": 2}[o.get("act")]
        self.emit(OPC_F16["PW"], [ib, ob, rb], tl, list(shp) + [h_in * w_in, ld, act, ldo, ow, opad, ldr], o)
        self.vbuf[o["out"]] = ob
        return i + 1

    def l_dwconv(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        _, h, w, c, _, _, _ = self.bufs[ib]
        ho, wo = self.vshape[o["out"]]
        self.bufs.append((F32, 1, 1, c, c, 0, c))
        cs = len(self.bufs) - 1
        ob = self.buf(F16, ho, wo, c)
        w9 = o["w"][:, 0].transpose(1, 2, 0).reshape(9, c)
        tl = [self.tensor(f"f16/dw.{k}.w", w9.astype(np.float16)),
              self.tensor(f"f16/dw.{k}.b", o["b"].astype(np.float16))]
        pt, pl = o["pads"][0], o["pads"][1]
        self.emit(OPC_F16["DW3"], [ib, ob, cs], tl, [h, w, c, o["s"][0], ho, wo, pt, pl], o)
        self.vbuf[o["out"]] = ob
        self.chsum = (ob, cs)
        return i + 1

    def l_se(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        cs = self.chsum[1]
        _, h, w, c, _, _, _ = self.bufs[ib]
        rd = o["w1"].shape[0]
        tl = [self.tensor(f"f16/se.{k}.w1", o["w1"]), self.tensor(f"f16/se.{k}.b1", o["b1"]),
              self.tensor(f"f16/se.{k}.w2t", np.ascontiguousarray(o["w2"].T)),
              self.tensor(f"f16/se.{k}.b2", o["b2"])]
        self.emit(OPC_F16["SE"], [ib, cs], tl, [c, rd, h * w], o)
        self.vbuf[o["out"]] = ib
        return i + 1

    def l_affine(self, i, o, k):
        nx, mn = self.ops[i + 1], self.ops[i + 2]
        ib = self.vbuf[o["ins"][0]]
        w = nx["w"].transpose(0, 2, 3, 1).reshape(1024, 1728)
        tl, shp = self.gemm_tensors(f"pc.{k}", w, nx["b"], 1728)
        tl = [self.tensor(f"f16/post.{k}.s", o["s"]), self.tensor(f"f16/post.{k}.t", o["t"])] + tl
        fb = self.buf(F32, 1, 1, 1024)
        pin = self.buf(F16, 8, 1, 1728)
        pout = self.buf(F16, 8, 1, 1024)
        self.emit(OPC_F16["POSTPC"], [ib, fb, pin, pout], tl, list(shp), o)
        self.vbuf[mn["out"]] = fb
        return i + 3

    def l_dense(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        n = o["w"].shape[0]
        ob = self.buf(F32, 1, 1, n)
        if n > 64:  # the compiler's default policy: an fp16 head above 64 classes
            tl = [self.tensor(f"f16/dense.{k}.w", o["w"].astype(np.float16)), self.tensor(f"f16/dense.{k}.b", o["b"])]
            self.emit(OPC_F16["DENSE"], [ib, ob], tl, [n], o)
        else:  # small heads: the exact fp32 GEMV (variant 0) on both paths
            tl = [self.tensor(f"f32/dense.{k}.w", o["w"].astype(np.float32)), self.tensor(f"f32/dense.{k}.b", o["b"])]
            self.emit(OPC_DENSE_F32, [ib, ob], tl, [n], o)
        self.vbuf[o["out"]] = ob
        return i + 1


def plan_slots(bufs, records, pinned):
    """Memory slots: buffers with disjoint op lifetimes and one dtype share a slot (best fit); buffer 0 and the pinned
    outputs get their own (lower.py plan_slots rules)."""
    first, last = {}, {}
    for i, (_, bl, _, _) in enumerate(records):
        for b in bl:
            if b >= 0:
                first.setdefault(b, i)
                last[b] = i
    esz = {0: 4, 1: 2, 2: 1, 3: 4}
    slot = {0: 0}
    slots = [None]
    for b in pinned:
        if b is not None and b not in slot:
            slot[b] = len(slots)
            slots.append([bufs[b][0], 0, 1 << 30])
    for i, (_, bl, _, _) in enumerate(records):
        for b in bl:
            if b < 0 or b in slot or first[b] != i:
                continue
            need = bufs[b][6] * esz[bufs[b][0]]
            free = [j for j in range(1, len(slots)) if slots[j][0] == bufs[b][0] and slots[j][2] < i]
            if not free:
                slots.append([bufs[b][0], 0, 0])
                j = len(slots) - 1
            else:
                fit = [j for j in free if slots[j][1] >= need]
                j = min(fit, key=lambda s: slots[s][1]) if fit else max(free, key=lambda s: slots[s][1])
            slots[j][1] = max(slots[j][1], need)
            slots[j][2] = last[b]
            slot[b] = j
    for b in range(len(bufs)):
        if b not in slot:
            slot[b] = len(slots)
            slots.append([bufs[b][0], 0, 0])
    return [tuple(bufs[b]) + (slot[b],) for b in range(len(bufs))]


# ------------------------------------------------------------------ the .bnpk writer (pkgfmt.py:1-22 format)

_DT = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.int8): 2, np.dtype(np.int32): 3}


def _pad8(b):
    return b + b"\0" * ((8 - len(b) % 8) % 8)


def _meta(k, v):
    kb = k.encode()
    if isinstance(v, (bytes, bytearray)):
        ty, vb = 3, bytes(v)
    elif isinstance(v, (bool, int, np.integer)):
        ty, vb = 1, struct.pack("<q", int(v))
    elif isinstance(v, float):
        ty, vb = 2, struct.pack("<d", v)
    else:
        ty, vb = 0, str(v).encode()
    return _pad8(struct.pack("<HHI", len(kb), ty, len(vb)) + kb + vb)


def _record(code, bl, tl, il):
    body = struct.pack(f"<{len(bl) + len(tl) + len(il)}i", *(list(bl) + list(tl) + list(il)))
    rec = _pad8(struct.pack("<6H", code, 0, len(bl), len(tl), len(il), 0) + body)
    return rec[:2] + struct.pack("<H", len(rec)) + rec[4:]


def write_package(dst, meta, tensors, paths):
    """Writes a .bnpk: meta [(key, value)], tensors [(name, array)], paths [(name, hwcap, bufs, records, in, out,
    emb)]. Returns the file size."""
    mb = b"".join(_meta(k, v) for k, v in meta)
    meta_off = 64
    tensor_off = meta_off + len(mb)
    path_off = tensor_off + 96 * len(tensors)
    off = path_off + 72 * len(paths)
    pdesc, pblobs = [], []
    for name, hw, bufs, recs, ib, ob, eb in paths:
        bb = b"".join(struct.pack("<8IQ", *b[:6], b[7], 0, b[6]) for b in bufs)
        rb = b"".join(_record(*r) for r in recs)
        boff, ooff = off, off + len(bb)
        off = ooff + len(rb)
        pblobs += [bb, rb]
        pdesc.append(name.encode().ljust(24, b"\0") + struct.pack(
            "<8I2Q", hw, len(bufs), len(recs), len(rb), ib, ob, 0xffffffff if eb is None else eb, 0, boff, ooff))
    off = (off + 63) & ~63
    tdesc, tblobs = [], []
    for name, a in tensors:
        dims = list(a.shape) + [0] * (4 - a.ndim)
        tdesc.append(name.encode().ljust(48, b"\0") + struct.pack("<II4IQQQ", _DT[a.dtype], a.ndim, *dims, off,
                                                                  a.nbytes, 0))
        tblobs.append((off, a))
        off = (off + a.nbytes + 64 + 63) & ~63
    size = off + 64
    with open(dst, "wb") as f:
        f.write(b"BNNPKG01" + struct.pack("<IHH4I4Q", 0x01020304, 1, 1, len(meta), len(tensors), len(paths), 0,
                                          meta_off, tensor_off, path_off, size))
        f.write(mb)
        f.write(b"".join(tdesc))
        f.write(b"".join(pdesc))
        for b in pblobs:
            f.write(b)
        for o, a in tblobs:
            f.write(b"\0" * (o - f.tell()))
            f.write(a.tobytes())
        f.write(b"\0" * (size - f.tell()))
    return size


def write_int8_package(dst, ir):
    """Lowers v24_ir()'s result for the neon-int8 path and writes the package; returns (n_classes, emb_dim)."""
    ops, vshape, logits, feat = ir
    lw = _Int8Lowering(ops)
    lw.vshape = vshape
    lw.run()
    ob, eb = lw.vbuf[logits], lw.vbuf[feat]
    n_classes, emb_dim = lw.bufs[ob][3], lw.bufs[eb][3]
    bufs = plan_slots(lw.bufs, lw.records, [ob, eb])
    meta = [(f"src_nodes/{PATH}", "\n".join(lw.src))] + metadata(n_classes, emb_dim, labels_for(n_classes))
    write_package(dst, meta, lw.tensors, [(PATH, 0, bufs, lw.records, 0, ob, eb)])
    return n_classes, emb_dim


def write_f16_package(dst, ir):
    """Lowers v24_ir()'s result for the neon-fp16 path (bnc.py compile --paths neon-fp16) and writes the package;
    returns (n_classes, emb_dim)."""
    ops, vshape, logits, feat = ir
    lw = _F16Lowering(ops)
    lw.vshape = vshape
    lw.run()
    ob, eb = lw.vbuf[logits], lw.vbuf[feat]
    n_classes, emb_dim = lw.bufs[ob][3], lw.bufs[eb][3]
    bufs = plan_slots(lw.bufs, lw.records, [ob, eb])
    meta = [(f"src_nodes/{PATH_F16}", "\n".join(lw.src))] + metadata(n_classes, emb_dim, labels_for(n_classes))
    write_package(dst, meta, lw.tensors, [(PATH_F16, 1, bufs, lw.records, 0, ob, eb)])
    return n_classes, emb_dim


def make_package(dst, seed=0, mini=False, n_classes=None, path=PATH):
    """A synthetic v2.4-architecture package (path "neon-int8" or "neon-fp16") at dst; returns (n_classes,
    emb_dim)."""
    nc = n_classes if n_classes is not None else (61 if mini else 6522)
    ir = v24_ir(seed, nc, MINI_BLOCKS if mini else V24_BLOCKS)
    return (write_f16_package if path == PATH_F16 else write_int8_package)(dst, ir)


# ------------------------------------------------------------------ the int8 prototype head (PROTO_S8)

OPC_PROTO_S8 = 35
PERCH_SAMPLE_RATE = 32000
BNN_MODEL_PERCH_V2 = 120
BNN_MODEL_BIRDNET_V3 = 30


def quant_rows_s8(w):
    """Per-row symmetric int8 of a float32 [N][K] matrix, as lower.py quant_rows_s8: sw = max |row| / 127 (0 for a
    zero row), q = round half away from zero of w / sw clipped to [-127, 127], in float32 arithmetic."""
    am = np.abs(w).max(1)
    sw = np.where(am > 0, am / 127.0, 0.0).astype(np.float32)
    sw_safe = np.where(sw > 0, sw, 1)
    q = np.where(sw[:, None] > 0, w / sw_safe[:, None], 0)
    q = np.clip(np.sign(q) * np.floor(np.abs(q) + 0.5), -127, 127).astype(np.int8)
    return q, sw


N4_LANE_LIMIT = 258


def n4_panel_flags(q):
    """One flag per 4-row panel of int8 [Np][Kp] weights: 1 where every int16 lane of the reference's n=4 K loop (bytes
    l, l + 8, l + 16, l + 24 of each 32-byte step) has sum |w| <= 258; all 0 when Kp % 32 != 0 (lower.py
    n4_panel_flags)."""
    rows, kp = q.shape
    if kp % 32:
        return np.zeros(rows // 4, np.int8)
    lane = np.abs(q.astype(np.int32)).reshape(rows, kp // 32, 4, 8).sum(2)
    worst = lane.max(axis=(1, 2))
    return (worst.reshape(rows // 4, 4).max(1) <= N4_LANE_LIMIT).astype(np.int8)


def proto_head(seed, n_cells, channels, n_classes, ppc, eps=1e-6, scale=1.0):
    """A seeded prototype head: prototypes [n_classes * ppc][channels] N(0, scale), class weights [n_classes][ppc]
    N(1, 0.1), class biases N(0, 0.05)."""
    rng = np.random.default_rng(seed)
    n = n_classes * ppc
    protos = (rng.standard_normal((n, channels)) * scale).astype(np.float32)
    cw = (1.0 + 0.1 * rng.standard_normal((n_classes, ppc))).astype(np.float32)
    cb = (0.05 * rng.standard_normal(n_classes)).astype(np.float32)
    return dict(P=protos, cw=cw, cb=cb, eps=float(eps), n_cells=int(n_cells))


def pack_proto_s8(protos):
    """The neon-int8 prototype tensors (lower.py proto_s8n): q [Np/4][Kp/16][4][16] int8 (Np = N rounded up to 4,
    Kp = K rounded up to 16, zero padding), sw [Np], n4 [Np/4]; also returns the unpacked q [Np][Kp]."""
    n, c = protos.shape
    n_pad, k_pad = (n + 3) & ~3, _r16(c)
    wq = np.zeros((n_pad, k_pad), np.float32)
    wq[:n, :c] = protos
    q, sw = quant_rows_s8(wq)
    qp = q.reshape(n_pad // 4, 4, k_pad // 16, 16).transpose(0, 2, 1, 3).copy()
    return qp, sw, n4_panel_flags(q), q


def pack_proto_s8_sdot(protos):
    """The neon-fp16 path's SDOT prototype tensors (lower.py proto_s8, PROTO variant 2): q [Np/12][K/4][12][4] int8
    (Np = N rounded up to 12, zero rows), sw [Np]; also returns the unpacked q [Np][K]. K % 4 == 0."""
    n, c = protos.shape
    n_pad = (n + 11) // 12 * 12
    wq = np.zeros((n_pad, c), np.float32)
    wq[:n] = protos
    q, sw = quant_rows_s8(wq)
    qp = q.reshape(n_pad // 12, 12, c // 4, 4).transpose(0, 2, 1, 3).copy()
    return qp, sw, q


def write_proto_package(dst, head, ld=None, model_id="perch_v2_proto_head_synthetic"):
    """A one-op neon-int8 package: PROTO_S8 on the input window taken as cells [n_cells][ld] (the first C = K
    channels of each row used), logits [n_classes] out. Buffers, tensors, record and slots as the reference compiler
    makes them for a prototype head (lower.py proto_s8n / emit_proto / cls_tensors, plan_slots). Returns
    (n_classes, n_samples)."""
    protos = head["P"]
    n, c = protos.shape
    p_cells = head["n_cells"]
    ld = ld or c
    nc, ppc = head["cw"].shape
    ns = p_cells * ld
    qp, sw, n4, _ = pack_proto_s8(protos)
    n_pad, k_pad = qp.shape[0] * 4, qp.shape[1] * 16
    lw = _Int8Lowering([])
    lw.bufs = [(F32, 1, 1, ns, ns, 0, ns)]
    tl = [lw.tensor("s8n/proto.0.q", qp), lw.tensor("s8n/proto.0.s", sw), lw.tensor("s8n/proto.0.n4", n4),
          lw.tensor("cls.0.w", head["cw"]), lw.tensor("cls.0.b", head["cb"]),
          lw.tensor("cls.0.eps", np.array([head["eps"]], np.float32))]
    ob = lw.buf(F32, 1, 1, nc)
    ab = lw.buf(I8, p_cells, 1, k_pad)
    cm = lw.buf(F32, 1, 1, n_pad)
    lw.emit(OPC_PROTO_S8, [0, ob, ab, cm], tl, [n, c, k_pad, n_pad, p_cells, c, ld, nc, ppc], {})
    bufs = plan_slots(lw.bufs, lw.records, [ob])
    meta = [(f"src_nodes/{PATH}", "\n".join(lw.src))] + metadata(
        nc, 0, labels_for(nc), model_id=model_id, family=BNN_MODEL_PERCH_V2, sample_rate=PERCH_SAMPLE_RATE,
        n_samples=ns, attribution="synthetic prototype head (random weights)")
    write_package(dst, meta, lw.tensors, [(PATH, 0, bufs, lw.records, 0, ob, None)])
    return nc, ns


def cells(n, n_cells, ld, seed=0, scale=1.0):
    """n windows of cells [n][n_cells][ld] float32, N(0, scale) (a prototype head's input), window w seeded by
    (seed, w)."""
    out = np.empty((n, n_cells, ld), np.float32)
    for i in range(n):
        out[i] = np.random.default_rng((seed, i)).standard_normal((n_cells, ld)) * scale
    return out


# ------------------------------------------------------------------ the framed log-mel front end (FE_LOGMEL)

OPC_FE_LOGMEL = 8
# Perch-like geometry (32 kHz, 5 s windows; 20 ms frames, 10 ms hop, 1024-point FFT, 128 mel bins): the real Perch
# constants come from its ONNX graph, which is not available here
PERCH_FE = dict(nsamp=160000, frame=640, hop=320, pad=0, nfft=1024, nmel=128, fmin=60.0, fmax=16000.0,
                floor=1e-5, scale=1.0)


def logmel_frontend(nsamp, frame, hop, pad, nfft, nmel, fmin=60.0, fmax=None, floor=1e-5, scale=1.0,
                    rate=PERCH_SAMPLE_RATE):
    """A log-mel front end: periodic Hann window of `frame` samples, triangular mel filters up to fmax (default
    Nyquist) at `rate`."""
    fmax = fmax or rate / 2.0
    return dict(nsamp=nsamp, frame=frame, hop=hop, pad=pad, nfft=nfft, window=_hann(frame),
                mel=_mel_bank(nfft, fmin, fmax, nmel, rate), floor=float(floor), scale=float(scale))


def logmel_frames(fe):
    return (fe["nsamp"] + 2 * fe["pad"] - fe["frame"]) // fe["hop"] + 1


def write_logmel_package(dst, fe, model_id="perch_v2_frontend_synthetic"):
    """A one-op neon-int8 package: FE_LOGMEL on the input window, the spectrogram [frames][nmel] out (as lower.py
    l_fe_logmel writes the op: tensors fe/window, fe/mel, fe/consts; buffer [frames][nmel]). n_classes in the
    metadata is the spectrogram's size. Returns (frames, nmel)."""
    nmel = fe["mel"].shape[0]
    nfr = logmel_frames(fe)
    lw = _Int8Lowering([])
    lw.bufs = [(F32, 1, 1, fe["nsamp"], fe["nsamp"], 0, fe["nsamp"])]
    tl = [lw.tensor("fe/window", fe["window"]), lw.tensor("fe/mel", fe["mel"]),
          lw.tensor("fe/consts", np.array([fe["floor"], fe["scale"]], np.float32))]
    ob = lw.buf(F32, nfr, nmel, 1)
    lw.emit(OPC_FE_LOGMEL, [0, ob], tl, [fe["nsamp"], fe["frame"], fe["hop"], fe["pad"], fe["nfft"], nmel], {})
    bufs = plan_slots(lw.bufs, lw.records, [ob])
    n_out = nfr * nmel
    meta = [(f"src_nodes/{PATH}", "\n".join(lw.src))] + metadata(
        n_out, 0, labels_for(n_out), model_id=model_id, family=BNN_MODEL_PERCH_V2, sample_rate=PERCH_SAMPLE_RATE,
        n_samples=fe["nsamp"], attribution="synthetic log-mel front end")
    write_package(dst, meta, lw.tensors, [(PATH, 0, bufs, lw.records, 0, ob, None)])
    return nfr, nmel


# ------------------------------------------------------------------ the dB-image front end (FE_DBIMG)

OPC_FE_DBIMG = 16
DB_PAD_MODES = {"none": 0, "reflect": 1, "zero": 2}
# a BirdNET-v3.0-like geometry (the v3.0 model is not in this repository: its documented front end is reflect
# padding, a framed DFT, power, mel, dB with a top-db floor, min/max normalisation, a bilinear resize to 224 x 468 and
# three normalised channels, on 5 s windows at 32 kHz); the n_fft, hop, mel rows and constants here are stand-ins
V3_SAMPLE_RATE = 32000
V3_FE = dict(nsamp=160000, nfft=1024, hop=320, pad=512, pad_mode="reflect", nmel=128, rows=tuple(range(96)),
             Ho=224, Wo=468, C=3, top_db=80.0, norm=1, floor=1e-10, eps=1e-6)


def dbimg_frontend(nsamp, nfft, hop, pad, pad_mode, nmel, rows, Ho, Wo, C, top_db=80.0, norm=1, floor=1e-10,
                   eps=1e-6, post=None, chan=None, rate=V3_SAMPLE_RATE, fmin=0.0, fmax=None):
    """A dB-image front end: periodic Hann window of nfft samples, triangular mel filters up to fmax (default Nyquist),
    dB = 10 log10 (ln times 10 / ln 10), the given mel rows, and C channels normalised by a seeded mean and std
    (subtract, then divide)."""
    fmax = fmax or rate / 2.0
    if post is None:
        post = [(1, float(np.float32(10.0 / np.log(10.0))))]
    if chan is None:
        rng = np.random.default_rng(C)
        chan = [(4, rng.uniform(0.3, 0.6, C).astype(np.float32)), (2, rng.uniform(0.2, 0.3, C).astype(np.float32))]
    nfr = (nsamp + 2 * pad - nfft) // hop + 1
    return dict(nsamp=nsamp, nfft=nfft, hop=hop, pad=pad, pad_mode=pad_mode, nfr=nfr, window=_hann(nfft),
                mel=_mel_bank(nfft, fmin, fmax, nmel, rate), rows=np.array(rows, np.int32), Ho=Ho, Wo=Wo, C=C,
                top_db=top_db, norm=norm, floor=float(floor), eps=float(eps), post=list(post), chan=list(chan))


def dbimg_record(fe, halo=0):
    """(tensors {name: array}, ints, ld, halo) of FE_DBIMG as lower.py l_fe_dbimg writes them (halo 0: an image whose
    consumers take none; a dense conv consumer takes a zero halo)"""
    c = fe["C"]
    ld, h = (c if c % 4 == 0 else (c + 3) & ~3), halo
    post = list(fe["post"]) + [(0, 0.0)] * (3 - len(fe["post"]))
    chan = list(fe["chan"]) + [(0, np.zeros(c, np.float32))] * (2 - len(fe["chan"]))
    scalars = np.array([fe["floor"], fe["top_db"] or 0.0, fe["eps"]] + [v for _, v in post], np.float32)
    consts = np.concatenate([scalars, np.asarray(chan[0][1], np.float32).reshape(-1),
                             np.asarray(chan[1][1], np.float32).reshape(-1)])
    ints = [fe["nsamp"], fe["nfft"], fe["hop"], fe["pad"], DB_PAD_MODES[fe["pad_mode"]], fe["nfr"], fe["mel"].shape[0],
            len(fe["rows"]), int(fe["top_db"] is not None), fe["norm"], post[0][0], post[1][0], post[2][0], 1,
            fe["Ho"], fe["Wo"], c, chan[0][0], chan[1][0], ld, h]
    tens = {"window": fe["window"], "mel": fe["mel"], "rows": np.asarray(fe["rows"], np.int32), "consts": consts}
    return tens, ints, ld, h


def write_dbimg_package(dst, fe, model_id="birdnet_v3_frontend_synthetic", halo=0):
    """A one-op neon-int8 package: FE_DBIMG on the input window, the image [Ho + 2 halo][Wo + 2 halo][ld] out (as
    lower.py l_fe_dbimg writes the op: tensors fe/dbimg.0.{window, mel, rows, consts}; buffer Ho x Wo x C, channel
    stride ld, the halo zero). n_classes in the metadata is the image's size. Returns the image's elements."""
    tens, ints, ld, h = dbimg_record(fe, halo)
    lw = _Int8Lowering([])
    lw.bufs = [(F32, 1, 1, fe["nsamp"], fe["nsamp"], 0, fe["nsamp"])]
    tl = [lw.tensor(f"fe/dbimg.0.{k}", tens[k]) for k in ("window", "mel", "rows", "consts")]
    hw = (fe["Ho"] + 2 * h) * (fe["Wo"] + 2 * h) * ld
    ob = lw.buf(F32, fe["Ho"], fe["Wo"], fe["C"], ld=ld, halo=h, elems=hw + 24 * ld + 64 if h else None)
    lw.emit(OPC_FE_DBIMG, [0, ob], tl, ints, {})
    bufs = plan_slots(lw.bufs, lw.records, [ob])
    n_out = hw
    meta = [(f"src_nodes/{PATH}", "\n".join(lw.src))] + metadata(
        n_out, 0, labels_for(n_out), model_id=model_id, family=BNN_MODEL_BIRDNET_V3, sample_rate=V3_SAMPLE_RATE,
        n_samples=fe["nsamp"], attribution="synthetic dB-image front end")
    write_package(dst, meta, lw.tensors, [(PATH, 0, bufs, lw.records, 0, ob, None)])
    return n_out


def pack_f32(w, b, kp):
    """fp32 GEMM weights as the reference packs them (fp_pack, src/gemm_f32.c:22-34): panels [Np/8][Kp][8] (+ slack)
    and the bias [Np + 8]; returns (panels, bias, (N, K, Kp, Np))"""
    return _Int8Lowering.pack_f32(np.asarray(w, np.float32), np.asarray(b, np.float32), kp)


def write_ops_package(dst, bufs, tensors, records, out_buf, emb_buf=None, model_id="op_test_synthetic",
                      family=BNN_MODEL_BIRDNET_V3, sample_rate=V3_SAMPLE_RATE, nodes=None):
    """A neon-int8 package of the given op records, for op-level tests: bufs [(dtype, H, W, C, ld, halo, elems)] with
    buffer 0 the input window (n_samples = its elems: an op reads the window in the layout buffer 0 declares),
    tensors [(name, array)], records [(code, bufs, tensors, ints)]; n_classes and emb_dim in the metadata are the
    output and embedding buffers' elements. Returns (n_classes, emb_dim)."""
    pinned = [out_buf] + ([emb_buf] if emb_buf is not None else [])
    bplan = plan_slots(bufs, records, pinned)
    n_out, n_emb = bufs[out_buf][6], bufs[emb_buf][6] if emb_buf is not None else 0
    names = nodes or [f"op{i}" for i in range(len(records))]
    meta = [(f"src_nodes/{PATH}", "\n".join(f"'{n}'" for n in names))] + metadata(
        n_out, n_emb, labels_for(n_out), model_id=model_id, family=family, sample_rate=sample_rate,
        n_samples=bufs[0][6], attribution="synthetic op test")
    write_package(dst, meta, list(tensors), [(PATH, 0, bplan, records, 0, out_buf, emb_buf)])
    return n_out, n_emb


# ------------------------------------------------------------------ a Perch-v2-architecture model (neon-fp16 + int8 head)

OPC_PERCH = dict(STEM=0x109, DWK=0x10a, PAD=0x10b, MEAN=0x10c, PROTO_F16S8=0x20d)
# the EfficientNet-B3 stages of Perch v2's backbone (results/perch_graph_compact.txt, results/perch_mac_table.txt):
# (blocks, depthwise k, first block's stride and pads [top, left, bottom, right], c_in, expansion, c_out)
PERCH_STAGES = ((2, 3, 1, [1, 1, 1, 1], 40, 1, 24), (3, 3, 2, [1, 1, 1, 1], 24, 6, 32),
                (3, 5, 2, [2, 1, 2, 2], 32, 6, 48), (5, 3, 2, [1, 0, 1, 1], 48, 6, 96),
                (5, 5, 1, [2, 2, 2, 2], 96, 6, 136), (6, 5, 2, [1, 1, 2, 2], 136, 6, 232),
                (2, 3, 1, [1, 1, 1, 1], 232, 6, 384))
# one block per stage, but both blocks of the first and the last stage: every op kind and geometry of the full
# model (DW3 on the stem output, PAD + DWK k3 of an unexpanded residual block, every strided depthwise form, DWK k3
# above 2048 channels)
PERCH_MINI_COUNTS = (2, 1, 1, 1, 1, 1, 2)
PERCH_MINI_FE = dict(PERCH_FE, nsamp=80000)  # 249 frames: 124 x 63 after the stem, 8 x 4 cells
PERCH_STEM = 40
PERCH_TOP = 1536
PERCH_HEAD = (14795, 4)  # classes x prototypes per class: 59180 prototypes (results/perch_graph_compact.txt:1129-1135)


def perch_ir(seed=0, mini=False, n_classes=None, ppc=None, fe=None):
    """The fused IR of a Perch-v2-architecture model with seeded random weights: FE_LOGMEL (a Perch-like log-mel
    front end), the 3x3 stride-2 stem, 26 MBConv blocks (SE on every block) in the stages of PERCH_STAGES, the
    1x1 top conv to 1536 channels, the prototype head on the 16 x 4 cells and the spatial mean (the embedding).
    mini: one block per inner stage (PERCH_MINI_COUNTS), 61 classes and 2.5 s windows (8 x 4 cells), for tests.

    Returns:
        (ops, vshape, logits_value, embedding_value, fe)
    """
    rng = np.random.default_rng(seed)
    f32 = np.float32
    nc = n_classes if n_classes is not None else (61 if mini else PERCH_HEAD[0])
    ppc = ppc or PERCH_HEAD[1]
    fe = fe or logmel_frontend(**(PERCH_MINI_FE if mini else PERCH_FE))

    def he(*shape, fan_in, scale=1.0):
        return (rng.standard_normal(shape) * (scale * np.sqrt(2.0 / fan_in))).astype(f32)

    def bias(n, sd=0.02):
        return (rng.standard_normal(n) * sd).astype(f32)

    ops, vshape = [], {}
    nid = [0]

    def val(h, w):
        nid[0] += 1
        vshape[nid[0]] = (h, w)
        return nid[0]

    nmel = fe["mel"].shape[0]
    h, w = logmel_frames(fe), nmel
    spec = val(h, w)
    ops.append(dict(op="FE_LOGMEL", ins=[], out=spec, fe=fe, nodes=["perch/frontend"]))
    h, w = (h - 3) // 2 + 1, (w - 3) // 2 + 1
    x = val(h, w)
    ops.append(dict(op="CONV", ins=[spec], out=x, w=he(PERCH_STEM, 1, 3, 3, fan_in=9), b=bias(PERCH_STEM), k=[3, 3],
                    s=[2, 2], pads=[0, 0, 0, 0], act="swish", nodes=["perch/stem"]))
    blk = 0
    for si, (n, k, st0, pads0, cin0, ex, cout) in enumerate(PERCH_STAGES):
        for j in range(PERCH_MINI_COUNTS[si] if mini else n):
            cin = cin0 if j == 0 else cout
            st = st0 if j == 0 else 1
            pads = pads0 if j == 0 else [(k - 1) // 2] * 4
            cm = cin * ex
            rd = max(1, cin // 4)
            tag = f"perch/block{blk}"
            e = x
            if ex != 1:
                e = val(h, w)
                ops.append(dict(op="CONV", ins=[x], out=e, w=he(cm, cin, 1, 1, fan_in=cin), b=bias(cm), k=[1, 1],
                                s=[1, 1], pads=[0, 0, 0, 0], act="swish", nodes=[f"{tag}/expand"]))
            ho = (h + pads[0] + pads[2] - k) // st + 1
            wo = (w + pads[1] + pads[3] - k) // st + 1
            d = val(ho, wo)
            ops.append(dict(op="DWCONV", ins=[e], out=d, w=he(cm, 1, k, k, fan_in=k * k), b=bias(cm), k=[k, k],
                            s=[st, st], pads=list(pads), act="swish", nodes=[f"{tag}/dw"]))
            g = val(ho, wo)
            ops.append(dict(op="SE", ins=[d], out=g, w1=he(rd, cm, fan_in=cm), b1=bias(rd), act1="swish",
                            w2=he(cm, rd, fan_in=rd), b2=bias(cm, 0.5), nodes=[f"{tag}/se"]))
            y = val(ho, wo)
            proj = dict(op="CONV", ins=[g], out=y, w=he(cout, cm, 1, 1, fan_in=cm, scale=0.35), b=bias(cout),
                        k=[1, 1], s=[1, 1], pads=[0, 0, 0, 0], act=None, nodes=[f"{tag}/project"])
            if st == 1 and cin == cout:
                proj["res"] = x
            ops.append(proj)
            x, h, w = y, ho, wo
            blk += 1
    top = val(h, w)
    c_last = PERCH_STAGES[-1][6]
    ops.append(dict(op="CONV", ins=[x], out=top, w=he(PERCH_TOP, c_last, 1, 1, fan_in=c_last), b=bias(PERCH_TOP),
                    k=[1, 1], s=[1, 1], pads=[0, 0, 0, 0], act="swish", nodes=["perch/top"]))
    head = proto_head(seed + 1, h * w, PERCH_TOP, nc, ppc, scale=1.0)
    logits = val(1, 1)
    ops.append(dict(op="PROTO", ins=[top], out=logits, P=head["P"], cw=head["cw"], cb=head["cb"], eps=head["eps"],
                    nodes=["perch/protopnet"]))
    emb = val(1, 1)
    ops.append(dict(op="MEAN", ins=[top], out=emb, nodes=["perch/embedding"]))
    return ops, vshape, logits, emb, fe


class _PerchF16Lowering(_F16Lowering):
    """The neon-fp16 lowering of a compiled model's IR with the int8 SDOT prototype head (bnc.py compile --paths
    neon-fp16 --proto-s8), for the op kinds of Perch v2. Follows python/bnneon/compiler/lower.py: l_fe_logmel, stem
    (im2col fp32 GEMM to fp16), pw / out_for_dw (a zero halo of (k - 1) / 2 for a lone depthwise consumer),
    l_dwconv / dw_input (DW3 for a 3x3 on a halo-1 buffer with pads <= 1 and C <= 2048, else PAD when needed + DWK),
    l_se (in place), l_mean, proto_s8 / emit_proto / cls_tensors."""

    def __init__(self, ops, nsamp):
        super().__init__(ops)
        self.bufs = [(F32, 1, 1, nsamp, nsamp, 0, nsamp)]

    def l_fe_logmel(self, i, o, k):
        fe = o["fe"]
        nmel = fe["mel"].shape[0]
        tl = [self.tensor("fe/window", fe["window"]), self.tensor("fe/mel", fe["mel"]),
              self.tensor("fe/consts", np.array([fe["floor"], fe["scale"]], np.float32))]
        ob = self.buf(F32, logmel_frames(fe), nmel, 1)
        self.emit(OPC_FE_LOGMEL, [0, ob], tl, [fe["nsamp"], fe["frame"], fe["hop"], fe["pad"], fe["nfft"], nmel], o)
        self.vbuf[o["out"]] = ob
        return i + 1

    def out_for_dw(self, o, ho, wo, co):
        cons = self.uses.get(o["out"], [])
        if len(cons) == 1 and cons[0]["op"] == "DWCONV" and co % 8 == 0:
            hk = (cons[0]["k"][0] - 1) // 2
            return self.buf(F16, ho, wo, co, ld=co, halo=hk), wo, hk, co
        ldo = _r8(co)
        return self.buf(F16, ho, wo, co, ld=ldo), 0, 0, ldo

    def l_conv(self, i, o, k):
        w, b = o["w"], o["b"]
        co = w.shape[0]
        ib = self.vbuf[o["ins"][0]]
        dt, h_in, w_in, _, ld, _, _ = self.bufs[ib]
        if o["k"] != [1, 1]:  # the stem: dense k x k VALID conv on the 1-channel fp32 image
            kk, st = o["k"][0], o["s"][0]
            ho, wo = self.vshape[o["out"]]
            taps = kk * kk
            k_pad = (taps + 3) & ~3
            panels, bb, shp = self.pack_f32(w.reshape(co, taps), b, k_pad)
            tl = [self.tensor(f"f32/stem.{k}.w", panels), self.tensor(f"f32/stem.{k}.b", bb)]
            ob, _, opad, ldo = self.out_for_dw(o, ho, wo, co)
            col = self.buf(F32, _r8(ho * wo), 1, k_pad)
            tmp = self.buf(F32, ho * wo, 1, shp[3])
            act = {None: 0, "swish": 1, "relu": 2}[o.get("act")]
            self.emit(OPC_PERCH["STEM"], [ib, ob, col, tmp], tl,
                      list(shp) + [h_in, w_in, ho, wo, kk, st, act, ldo, opad], o)
            self.vbuf[o["out"]] = ob
            return i + 1
        tl, shp = self.gemm_tensors(f"pw.{k}", w[:, :, 0, 0], b, _r8(w.shape[1]))
        ob, ow, opad, ldo = self.out_for_dw(o, h_in, w_in, co)
        rb, ldr = -1, 0
        if o.get("res"):
            rb = self.vbuf[o["res"]]
            ldr = self.bufs[rb][4]
        act = {None: 0, "swish": 1, "relu": 2}[o.get("act")]
        self.emit(OPC_F16["PW"], [ib, ob, rb], tl, list(shp) + [h_in * w_in, ld, act, ldo, ow, opad, ldr], o)
        self.vbuf[o["out"]] = ob
        return i + 1

    def l_dwconv(self, i, o, k):
        kk, st, pads = o["k"][0], o["s"][0], o["pads"]
        ib = self.vbuf[o["ins"][0]]
        _, h, w, c, ld, halo, _ = self.bufs[ib]
        pt, pl, pb, pr = pads
        ho, wo = self.vshape[o["out"]]
        self.bufs.append((F32, 1, 1, c, c, 0, c))
        cs = len(self.bufs) - 1
        ob = self.buf(F16, ho, wo, c)
        w9 = o["w"][:, 0].transpose(1, 2, 0).reshape(kk * kk, c)
        if kk == 3 and halo == 1 and ld == c and max(pads) <= 1 and c <= 2048:
            tl = [self.tensor(f"f16/dw.{k}.w", w9.astype(np.float16)),
                  self.tensor(f"f16/dw.{k}.b", o["b"].astype(np.float16))]
            self.emit(OPC_F16["DW3"], [ib, ob, cs], tl, [h, w, c, st, ho, wo, pt, pl], o)
        else:
            hk = (kk - 1) // 2
            if halo != hk or ld != c:  # dw_input: a PAD into a buffer with halo hk and ld == C
                pb_ = self.buf(F16, h, w, c, ld=c, halo=hk)
                self.emit(OPC_PERCH["PAD"], [ib, pb_], [], [h, w, c, ld, hk], o)
                ib = pb_
            tl = [self.tensor(f"f16/dw.{k}.w", w9.astype(np.float16)),
                  self.tensor(f"f16/dw.{k}.b", o["b"].astype(np.float16))]
            self.emit(OPC_PERCH["DWK"], [ib, ob, cs], tl, [h, w, c, kk, st, pt, pl, ho, wo, 1], o)
        self.vbuf[o["out"]] = ob
        self.chsum = (ob, cs)
        return i + 1

    def l_mean(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        _, h, w, c, ld, _, _ = self.bufs[ib]
        ob = self.buf(F32, 1, 1, c)
        self.emit(OPC_PERCH["MEAN"], [ib, ob], [], [h * w, c, ld], o)
        self.vbuf[o["out"]] = ob
        return i + 1

    def l_proto(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        _, h, w, c, ld, _, _ = self.bufs[ib]
        n_proto = o["P"].shape[0]
        nc, ppc = o["cw"].shape
        qp, sw, _ = pack_proto_s8_sdot(o["P"])
        n_pad = qp.shape[0] * 12
        tl = [self.tensor(f"s8/proto.{k}.q", qp), self.tensor(f"s8/proto.{k}.s", sw),
              self.tensor(f"cls.{k}.w", o["cw"]), self.tensor(f"cls.{k}.b", o["cb"]),
              self.tensor(f"cls.{k}.eps", np.array([o["eps"]], np.float32))]
        ob = self.buf(F32, 1, 1, nc)
        ab = self.buf(I8, h * w, 1, c)
        cm = self.buf(F32, 1, 1, n_pad)
        self.emit(OPC_PERCH["PROTO_F16S8"], [ib, ob, ab, cm], tl, [n_proto, c, n_pad, h * w, c, ld, nc, ppc], o)
        self.vbuf[o["out"]] = ob
        return i + 1


def write_perch_package(dst, ir):
    """Lowers perch_ir()'s result for the neon-fp16 path with the int8 SDOT prototype head and writes the package
    (hwcap fp16 | dotprod, as the reference compiler sets it for a path with variant-2 ops); returns (n_classes,
    emb_dim, n_samples)."""
    ops, vshape, logits, emb, fe = ir
    lw = _PerchF16Lowering(ops, fe["nsamp"])
    lw.vshape = vshape
    lw.run()
    ob, eb = lw.vbuf[logits], lw.vbuf[emb]
    n_classes, emb_dim = lw.bufs[ob][3], lw.bufs[eb][3]
    bufs = plan_slots(lw.bufs, lw.records, [ob, eb])
    meta = [(f"src_nodes/{PATH_F16}", "\n".join(lw.src))] + metadata(
        n_classes, emb_dim, labels_for(n_classes), model_id="perch_v2_synthetic", family=BNN_MODEL_PERCH_V2,
        sample_rate=PERCH_SAMPLE_RATE, n_samples=fe["nsamp"],
        attribution="synthetic Perch-v2-architecture model (random weights)")
    write_package(dst, meta, lw.tensors, [(PATH_F16, 3, bufs, lw.records, 0, ob, eb)])
    return n_classes, emb_dim, fe["nsamp"]


class _PerchInt8Lowering(_Int8Lowering):
    """The neon-int8 lowering of a compiled model's IR for the op kinds of Perch v2 with the reference compiler's
    default int8 policy (lower.py INT8_DEFAULT "pw,head,sed,lin,proto"): 1x1 convs with an activation ("pw") and those
    feeding the mean ("head") on PW_S8, the projections ("pwl": no activation, SE-gated) on the fp32 PW, the int8
    prototype head PROTO_S8 (proto_s8n). Follows python/bnneon/compiler/lower.py: l_fe_logmel, stem (STEM variant 0:
    im2col + fp32 GEMM into the fp32 output), pw / int8_class / out_for_dw (a zero halo of (k - 1) / 2 for a lone
    depthwise consumer), l_dwconv / dw_input (DW3 for a 3x3 with pads 1 on a halo-1 buffer, else PAD when needed +
    DWK), l_se (SE_GATE, the gate applied by the next 1x1 conv), l_mean, proto_s8n / emit_proto / cls_tensors."""

    CLASSES = ("pw", "head", "sed", "lin", "proto")

    def __init__(self, ops, nsamp):
        super().__init__(ops)
        self.bufs = [(F32, 1, 1, nsamp, nsamp, 0, nsamp)]

    l_fe_logmel = _PerchF16Lowering.l_fe_logmel

    def out_buffer(self, o, ho, wo, co):
        cons = self.uses.get(o["out"], [])
        if len(cons) == 1 and cons[0]["op"] == "DWCONV" and co % 8 == 0:
            hk = (cons[0]["k"][0] - 1) // 2
            return self.buf(F32, ho, wo, co, ld=co, halo=hk), wo, hk, co
        ldo = _r8(co)
        return self.buf(F32, ho, wo, co, ld=ldo), 0, 0, ldo

    def int8_class(self, o):
        if any(c["op"] in ("GEM", "SED", "MEAN") for c in self.uses.get(o["out"], [])):
            return "head"
        return "pwl" if o.get("act") is None else "pw"

    def l_conv(self, i, o, k):
        w, b = o["w"], o["b"]
        co = w.shape[0]
        ib = self.vbuf[o["ins"][0]]
        _, h_in, w_in, _, ld, _, _ = self.bufs[ib]
        act = {None: 0, "swish": 1, "relu": 2}[o.get("act")]
        if o["k"] != [1, 1]:  # the stem: dense k x k VALID conv on the 1-channel fp32 image
            kk, st = o["k"][0], o["s"][0]
            ho, wo = self.vshape[o["out"]]
            k_pad = (kk * kk + 3) & ~3
            panels, bb, shp = self.pack_f32(w.reshape(co, kk * kk), b, k_pad)
            tl = [self.tensor(f"f32/stem.{k}.w", panels), self.tensor(f"f32/stem.{k}.b", bb)]
            ob, _, opad, ldo = self.out_buffer(o, ho, wo, co)
            col = self.buf(F32, _r8(ho * wo), 1, k_pad)
            self.emit(OPC_PERCH["STEM"] & 0xff, [ib, ob, col], tl, list(shp) + [h_in, w_in, ho, wo, kk, st, act, ldo, opad],
                      o)
            self.vbuf[o["out"]] = ob
            return i + 1
        w2 = w[:, :, 0, 0]
        s8 = self.int8_class(o) in self.CLASSES
        if s8:
            tl, shp = self.s8(f"pw.{k}", w2, b)
        else:
            panels, bb, shp = self.pack_f32(w2, b, _r8(w2.shape[1]))
            tl = [self.tensor(f"s8n/pw.{k}.w", panels), self.tensor(f"s8n/pw.{k}.b", bb)]
        ob, ow, opad, ldo = self.out_buffer(o, h_in, w_in, co)
        rb, ldr = -1, 0
        if o.get("res"):
            rb = self.vbuf[o["res"]]
            ldr = self.bufs[rb][4]
        gate = [self.gate[o["ins"][0]]] if o["ins"][0] in self.gate else []
        if s8:
            m4 = (h_in * w_in + 3) & ~3
            qb = self.buf(I8, m4, 1, shp[2])
            sb = self.buf(F32, m4, 1, 1)
            zb = self.buf(I32, m4, 1, 1)
            code, bl = OPC["PW_S8"], [ib, ob, rb, qb, sb, zb] + gate
        else:
            code, bl = OPC_PW_F32, [ib, ob, rb] + gate
        self.emit(code, bl, tl, list(shp) + [h_in * w_in, ld, act, ldo, ow, opad, ldr], o)
        self.vbuf[o["out"]] = ob
        return i + 1

    def l_dwconv(self, i, o, k):
        kk, st, pads = o["k"][0], o["s"][0], o["pads"]
        ib = self.vbuf[o["ins"][0]]
        _, h, w, c, ld, halo, _ = self.bufs[ib]
        pt, pl, _, _ = pads
        ho, wo = self.vshape[o["out"]]
        self.bufs.append((F32, 1, 1, c, c, 0, c))
        cs = len(self.bufs) - 1
        ob = self.buf(F32, ho, wo, c)
        w9 = o["w"][:, 0].transpose(1, 2, 0).reshape(kk * kk, c)
        tl = [self.tensor(f"s8n/dw.{k}.w", w9.astype(np.float32)),
              self.tensor(f"s8n/dw.{k}.b", o["b"].astype(np.float32))]
        if kk == 3 and halo == 1 and ld == c and max(pads) <= 1 and pt == 1 and pl == 1:
            self.emit(OPC["DW3"], [ib, ob, cs], tl, [h, w, c, st, ho, wo], o)
        else:
            hk = (kk - 1) // 2
            if halo != hk or ld != c:  # dw_input: a PAD into a buffer with halo hk and ld == C
                pb_ = self.buf(F32, h, w, c, ld=c, halo=hk)
                self.emit(OPC_PERCH["PAD"] & 0xff, [ib, pb_], [], [h, w, c, ld, hk], o)
                ib = pb_
            self.emit(OPC_PERCH["DWK"] & 0xff, [ib, ob, cs], tl, [h, w, c, kk, st, pt, pl, ho, wo, 1], o)
        self.vbuf[o["out"]] = ob
        self.chsum = (ob, cs)
        return i + 1

    def l_mean(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        _, h, w, c, ld, _, _ = self.bufs[ib]
        ob = self.buf(F32, 1, 1, c)
        self.emit(OPC_PERCH["MEAN"] & 0xff, [ib, ob], [], [h * w, c, ld], o)
        self.vbuf[o["out"]] = ob
        return i + 1

    def l_proto(self, i, o, k):
        ib = self.vbuf[o["ins"][0]]
        _, h, w, c, ld, _, _ = self.bufs[ib]
        n_proto = o["P"].shape[0]
        nc, ppc = o["cw"].shape
        qp, sw, n4, _ = pack_proto_s8(o["P"])
        n_pad, k_pad = qp.shape[0] * 4, qp.shape[1] * 16
        tl = [self.tensor(f"s8n/proto.{k}.q", qp), self.tensor(f"s8n/proto.{k}.s", sw),
              self.tensor(f"s8n/proto.{k}.n4", n4), self.tensor(f"cls.{k}.w", o["cw"]),
              self.tensor(f"cls.{k}.b", o["cb"]), self.tensor(f"cls.{k}.eps", np.array([o["eps"]], np.float32))]
        ob = self.buf(F32, 1, 1, nc)
        ab = self.buf(I8, h * w, 1, k_pad)
        cm = self.buf(F32, 1, 1, n_pad)
        self.emit(OPC_PROTO_S8, [ib, ob, ab, cm], tl, [n_proto, c, k_pad, n_pad, h * w, c, ld, nc, ppc], o)
        self.vbuf[o["out"]] = ob
        return i + 1


def write_perch_int8_package(dst, ir):
    """Lowers perch_ir()'s result for the neon-int8 path (the reference compiler's default int8 policy) and writes the
    package; returns (n_classes, emb_dim, n_samples)."""
    ops, vshape, logits, emb, fe = ir
    lw = _PerchInt8Lowering(ops, fe["nsamp"])
    lw.vshape = vshape
    lw.run()
    ob, eb = lw.vbuf[logits], lw.vbuf[emb]
    n_classes, emb_dim = lw.bufs[ob][3], lw.bufs[eb][3]
    bufs = plan_slots(lw.bufs, lw.records, [ob, eb])
    meta = [(f"src_nodes/{PATH}", "\n".join(lw.src))] + metadata(
        n_classes, emb_dim, labels_for(n_classes), model_id="perch_v2_synthetic", family=BNN_MODEL_PERCH_V2,
        sample_rate=PERCH_SAMPLE_RATE, n_samples=fe["nsamp"],
        attribution="synthetic Perch-v2-architecture model (random weights)")
    write_package(dst, meta, lw.tensors, [(PATH, 0, bufs, lw.records, 0, ob, eb)])
    return n_classes, emb_dim, fe["nsamp"]


def make_perch_package(dst, seed=0, mini=False, n_classes=None, ppc=None):
    """A synthetic Perch-v2-architecture neon-fp16 package with the int8 prototype head at dst; returns (n_classes,
    emb_dim, n_samples)."""
    return write_perch_package(dst, perch_ir(seed, mini, n_classes, ppc))


# ------------------------------------------------------------------ audio

def audio(n, seed=0, n_samples=NSAMP, rate=SAMPLE_RATE):
    """n windows [n][n_samples] float32: 0.1 N(0, 1) noise plus 1-3 linear chirps (1-12 kHz, amplitude 0.1-0.5,
    random start and length) per window, window w seeded by (seed, w), clipped to [-1, 1)."""
    out = np.empty((n, n_samples), np.float32)
    t = np.arange(n_samples) / rate
    for i in range(n):
        rng = np.random.default_rng((seed, i))
        x = 0.1 * rng.standard_normal(n_samples)
        for _ in range(int(rng.integers(1, 4))):
            f0, f1 = rng.uniform(1000.0, 12000.0, 2)
            amp = rng.uniform(0.1, 0.5)
            start = int(rng.integers(0, n_samples // 2))
            length = int(rng.integers(n_samples // 8, n_samples - start))
            tt = t[:length]
            ph = 2 * np.pi * (f0 * tt + 0.5 * (f1 - f0) / max(tt[-1], 1e-9) * tt * tt)
            x[start:start + length] += amp * np.sin(ph)
        out[i] = np.clip(x, -1.0, np.nextafter(np.float32(1.0), np.float32(0.0)))
    return out
