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
