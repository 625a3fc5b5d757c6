"""A minimal reader of the .bnpk op list (python/bnneon/compiler/pkgfmt.py layout) for the op-level tests."""
import struct

# buffer arguments each kernel writes (the reference registry's outmask) and the ones that are the int8 path's row
# scratch (q, sa, za), which the B200 runtime keeps in its own layout
# (fp16 ops: base | 1 << 8, the fp16 path's int8 prototype head base | 2 << 8; SE f16 scales its buffer 0 in place;
# POSTPC's im2col and GEMM rows stay in the runtime's own scratch, STEM f16 needs neither its im2col nor its fp32 rows)
OUTMASK = {1: 0x2, 2: 0x2, 3: 0x2, 4: 0x6, 9: 0x6, 10: 0x6, 11: 0x2, 12: 0x2, 16: 0x2, 17: 0x2, 18: 0x2, 19: 0x7E, 20: 0x4, 21: 0x2, 24: 0x3FE, 6: 0xE, 7: 0x2, 8: 0x2, 25: 0x2, 22: 0x3A, 23: 0x1E, 35: 0xE,
           0x102: 0x2, 0x103: 0x2, 0x104: 0x6, 0x105: 0x1, 0x106: 0xE, 0x107: 0x2,
           0x109: 0xE, 0x10A: 0x6, 0x10B: 0x2, 0x10C: 0x2, 0x20D: 0xE}
SCRATCH = {22: (3, 4, 5), 24: (7, 8, 9), 23: (2, 3, 4), 6: (2, 3), 35: (2,), 0x106: (2, 3), 0x109: (2, 3), 0x20D: (2,)}
NAMES = {1: "FE_STFT2", 2: "C0POOL", 3: "PW", 4: "DW3", 6: "POSTPC", 7: "DENSE", 8: "FE_LOGMEL", 9: "STEM", 10: "DWK", 11: "PAD", 12: "MEAN", 16: "FE_DBIMG", 17: "CONVK", 18: "GEM", 19: "SED",
         20: "VADD", 21: "CONVW", 24: "SED_S8", 22: "PW_S8", 23: "GEMV_S8",
         25: "SE_GATE", 35: "PROTO_S8", 0x102: "C0POOL_F16", 0x103: "PW_F16", 0x104: "DW3_F16", 0x105: "SE_F16",
         0x106: "POSTPC_F16", 0x107: "DENSE_F16", 0x109: "STEM_F16", 0x10A: "DWK_F16", 0x10B: "PAD_F16",
         0x10C: "MEAN_F16", 0x20D: "PROTO_F16S8"}


def read_ops(path, path_name="neon-int8"):
    """[(code, bufs, tensors, ints)] of the named path, and its buffer descriptors [(dtype, H, W, C, ld, halo, slot,
    elems)]."""
    with open(path, "rb") as f:
        data = f.read()
    _, _, n_paths, _ = struct.unpack_from("<4I", data, 16)
    _, _, path_off, _ = struct.unpack_from("<4Q", data, 32)
    for i in range(n_paths):
        o = path_off + 72 * i
        name = data[o:o + 24].rstrip(b"\0").decode()
        if name != path_name:
            continue
        _, n_buf, n_ops, _, _, _, _, _ = struct.unpack_from("<8I", data, o + 24)
        buf_off, ops_off = struct.unpack_from("<2Q", data, o + 56)
        bufs = []
        for b in range(n_buf):
            v = struct.unpack_from("<8IQ", data, buf_off + 40 * b)
            bufs.append((v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[8]))
        ops, q = [], ops_off
        for _ in range(n_ops):
            code, rec, nb, nt, ni, _ = struct.unpack_from("<6H", data, q)
            vals = struct.unpack_from(f"<{nb + nt + ni}i", data, q + 12)
            ops.append((code, list(vals[:nb]), list(vals[nb:nb + nt]), list(vals[nb + nt:])))
            q += rec
        return ops, bufs
    raise KeyError(path_name)


def op_io(code, bl):
    """(input buffer ids, output buffer ids) an op reads and writes, without the int8 row scratch."""
    mask, scratch = OUTMASK[code], SCRATCH.get(code, ())
    ins = [b for a, b in enumerate(bl) if b >= 0 and not (mask >> a & 1) and a not in scratch]
    outs = [b for a, b in enumerate(bl) if b >= 0 and (mask >> a & 1) and a not in scratch]
    return ins, outs


def op_offsets(path, path_name="neon-int8"):
    """File offsets of the op records of the named path (for tests that corrupt one record)."""
    with open(path, "rb") as f:
        data = f.read()
    _, _, n_paths, _ = struct.unpack_from("<4I", data, 16)
    _, _, path_off, _ = struct.unpack_from("<4Q", data, 32)
    for i in range(n_paths):
        o = path_off + 72 * i
        if data[o:o + 24].rstrip(b"\0").decode() != path_name:
            continue
        _, _, n_ops, _, _, _, _, _ = struct.unpack_from("<8I", data, o + 24)
        _, ops_off = struct.unpack_from("<2Q", data, o + 56)
        offs, q = [], ops_off
        for _ in range(n_ops):
            offs.append(q)
            q += struct.unpack_from("<H", data, q + 2)[0]
        return offs
    raise KeyError(path_name)


def tensor_offset(path, name):
    """File offset of the data of the tensor called `name` (for tests that corrupt one tensor)."""
    with open(path, "rb") as f:
        data = f.read()
    _, n_tensors, _, _ = struct.unpack_from("<4I", data, 16)
    _, tensor_off, _, _ = struct.unpack_from("<4Q", data, 32)
    for i in range(n_tensors):
        o = tensor_off + 96 * i
        if data[o:o + 48].rstrip(b"\0").decode() == name:
            return struct.unpack_from("<Q", data, o + 72)[0]
    raise KeyError(name)
