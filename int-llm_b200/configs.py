"""Workload definitions for the synthetic configurations (pure data, no compute).

Config indices follow the benchmark plan: 0 = TinyLlama greedy decode,
1 = M=1 matvec microbench, 2 = M=512 prefill GEMM, 3 = batched decode,
4 = Llama-2-7B shape. Model fields follow llama_config_t (llama_int.c:788-798).
Tensor names are the HuggingFace names llama_int loads (llama_int.c:1290-1298).
Synthetic tensors are seeded per tensor:
  seed = 0x494E544C4C4D0000 ^ (config << 32) ^ fnv1a64(name).
"""

# (dim, n_heads, n_kv_heads, head_dim, n_layers, inter, vocab, max_seq, rope_theta)
TINYLLAMA = dict(dim=2048, n_heads=32, n_kv_heads=4, head_dim=64, n_layers=22, inter=5632,
                 vocab=32000, max_seq=2048, rope_theta=10000)
LLAMA7B = dict(dim=4096, n_heads=32, n_kv_heads=32, head_dim=128, n_layers=32, inter=11008,
               vocab=32000, max_seq=2112, rope_theta=10000)
# small model with the same structure (GQA 4:1, SwiGLU), for fast parity tests
TINY_TEST = dict(dim=256, n_heads=8, n_kv_heads=2, head_dim=32, n_layers=2, inter=704,
                 vocab=512, max_seq=128, rope_theta=10000)

# Llama-2-7B geometry at reduced width for parity tests: head_dim 128, MHA
# (n_kv_heads = n_heads), FFN / dim = 11008 / 4096; positions beyond 384 reach
# the phased attention kernels
GEOM7B_TEST = dict(dim=512, n_heads=4, n_kv_heads=4, head_dim=128, n_layers=2, inter=1376,
                   vocab=1024, max_seq=448, rope_theta=10000)
# config-3 geometry (full TinyLlama width, GQA 8:1, head_dim 64) with 2 layers and a
# smaller vocabulary, decoding at context ~2100 with max_seq 2176
CFG3_TEST = dict(dim=2048, n_heads=32, n_kv_heads=4, head_dim=64, n_layers=2, inter=5632,
                 vocab=4096, max_seq=2176, rope_theta=10000)

# config 1: matvec shapes as (K, N) = (input length, output rows)
CFG1_SHAPES = [(2048, 2048), (2048, 256), (2048, 5632), (5632, 2048), (2048, 32000)]
# config 2: prefill GEMM M=512 on fused TinyLlama projections (K, N)
CFG2_ROWS = 512
CFG2_SHAPES = [("qkv", 2048, 2560), ("o", 2048, 2048), ("gate_up", 2048, 11264), ("down", 5632, 2048)]

LAYER_TENSORS = ["input_layernorm", "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                 "self_attn.o_proj", "post_attention_layernorm", "mlp.gate_proj", "mlp.up_proj",
                 "mlp.down_proj"]


def cfg9(c):
    return [c["dim"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["n_layers"], c["inter"],
            c["vocab"], c["max_seq"], c["rope_theta"]]


def layer_shapes(c):
    """Shapes of the 9 per-layer tensors in layer_weights_t order (llama_int.c:1250-1260)."""
    d, kv, it = c["dim"], c["n_kv_heads"] * c["head_dim"], c["inter"]
    return [(d,), (d, d), (kv, d), (kv, d), (d, d), (d,), (it, d), (it, d), (d, it)]


def layer_name(l, t):
    return f"model.layers.{l}.{t}.weight"


def matvec_names(K, N):
    return f"w:{K}x{N}", f"x:{K}x{N}"


def gemm_names(tag, K, N, rows):
    return f"w:{tag}:{K}x{N}", f"X:{rows}x{K}"
