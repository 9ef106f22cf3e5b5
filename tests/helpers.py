"""Shared test helpers: synthetic model weights from the oracle's generator."""
import numpy as np

import configs
import oracle as orc

ONE = 1 << 48


def model_weights(cfg_index, c):
    """Synthetic weights for a model config (all matrices seeded by tensor name;
    norm weights = 1.0 in Q16.48; untied LM head)."""
    d, V = c["dim"], c["vocab"]
    w = {"embed": orc.synth_weights(cfg_index, "model.embed_tokens.weight", (V, d)),
         "final_norm": np.full(d, ONE, dtype=np.int64),
         "lm_head": orc.synth_weights(cfg_index, "lm_head.weight", (V, d)),
         "layers": []}
    for l in range(c["n_layers"]):
        lay = []
        for t, shp in zip(configs.LAYER_TENSORS, configs.layer_shapes(c)):
            if len(shp) == 1:
                lay.append(np.full(shp, ONE, dtype=np.int64))
            else:
                lay.append(orc.synth_weights(cfg_index, configs.layer_name(l, t), shp))
        w["layers"].append(lay)
    return w


def layer_ptr_array(w):
    import ctypes
    ptrs = []
    for lay in w["layers"]:
        ptrs += [a.ctypes.data for a in lay]
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


class OracleModel:
    """The C restatement's model (iq_oracle.c) over numpy weights."""

    def __init__(self, c, w, lib=None, prefix="iqo_"):
        import ctypes
        self.c, self.w = c, w
        self.L = lib or orc.O
        self.pre = prefix
        self.cfg = (ctypes.c_int * 9)(*configs.cfg9(c))
        self.ptrs = layer_ptr_array(w)
        self.h = getattr(self.L, prefix + "model_create")(
            self.cfg, orc.p(w["embed"]), orc.p(w["final_norm"]), orc.p(w["lm_head"]), self.ptrs)

    def forward(self, tok, pos):
        lg = np.empty(self.c["vocab"], dtype=np.int64)
        a = getattr(self.L, self.pre + "model_forward")(self.h, tok, pos, orc.p(lg))
        return a, lg

    def reset(self):
        getattr(self.L, self.pre + "model_reset")(self.h)

    def generate(self, prompt, max_new):
        import ctypes
        pr = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(len(pr) + max_new, dtype=np.int32)
        if self.pre == "iqo_":
            lh = ctypes.c_uint64(0)
            n = self.L.iqo_model_generate(self.h, orc.p(pr), len(pr), max_new, orc.p(out),
                                          ctypes.byref(lh))
            return out[:n].tolist(), lh.value
        n = self.L.ref_model_generate(self.h, orc.p(pr), len(pr), max_new, orc.p(out))
        return out[:n].tolist(), None

    def close(self):
        getattr(self.L, self.pre + "model_free")(self.h)


# ------------------------------------------------------------ .mgw files

MGW_NAMES = {"embed": "model.embed_tokens.weight", "final_norm": "model.norm.weight",
             "lm_head": "lm_head.weight"}


def write_mgw(path, c, w, tied=False):
    """Writes a model in int-llm's native .mgw container (llama_int.c:386-454):
    64-byte header ("MGW\\0", version 1, endian tag 0x01020304, tensor count,
    index and data offsets), 64-byte config block (llama_config_t fields +
    lm_head_tied), 96-byte index entries (name[64], elements, offset, ndims,
    shape[2]), then 8-byte aligned little-endian int64 data."""
    import struct
    tensors = [(MGW_NAMES["embed"], w["embed"]), (MGW_NAMES["final_norm"], w["final_norm"])]
    if not tied:
        tensors.append((MGW_NAMES["lm_head"], w["lm_head"]))
    for l, lay in enumerate(w["layers"]):
        for t, a in zip(configs.LAYER_TENSORS, lay):
            tensors.append((configs.layer_name(l, t), a))
    n = len(tensors)
    index_off = 128
    data_off = index_off + 96 * n
    data_off = (data_off + 7) // 8 * 8
    hdr = struct.pack("<4sIIIQQ32s", b"MGW\0", 1, 0x01020304, n, index_off, data_off, b"\0" * 32)
    cfg = struct.pack("<10i24s", c["dim"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["n_layers"],
                      c["inter"], c["vocab"], c["max_seq"], c["rope_theta"], 1 if tied else 0, b"\0" * 24)
    idx, off = [], data_off
    for name, a in tensors:
        shp = list(a.shape) + [0] * (2 - a.ndim)
        idx.append(struct.pack("<64sQQIIII", name.encode(), a.size, off, a.ndim, shp[0], shp[1], 0))
        off += a.size * 8
    with open(path, "wb") as f:
        f.write(hdr + cfg + b"".join(idx))
        f.write(b"\0" * (data_off - f.tell()))
        for name, a in tensors:
            f.write(np.ascontiguousarray(a, dtype="<i8").tobytes())
