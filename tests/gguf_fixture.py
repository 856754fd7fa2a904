"""Write small GGUF files with gguf-py (the upstream writer) for the loader tests."""
import numpy as np

from thunderllamax_b200 import synth

TENSORS = [  # (name, qtype or numpy dtype, rows, k)
    ("blk.0.ffn_down.weight", "q6_k", 37, 512),
    ("blk.0.ffn_gate.weight", "iq3_xxs", 50, 768),
    ("blk.0.attn_v.weight", "q4_k", 16, 256),
    ("blk.0.attn_qkv.weight", "q5_k", 33, 512),
    ("blk.0.ssm_out.weight", "q8_0", 20, 512),
    ("blk.0.ffn_up_exps.weight", "iq4_xs", 18, 256),
    ("blk.0.attn_norm.weight", np.float32, 1, 96),
    ("blk.0.ssm_conv1d.weight", np.float32, 24, 4),
    ("token_embd_f16", np.float16, 5, 64),
]


def write_gguf(path, seed=0, alignment=None):
    import gguf
    rng = np.random.default_rng(seed)
    w = gguf.GGUFWriter(str(path), "qwen35")
    if alignment:
        w.add_custom_alignment(alignment)
    w.add_uint32("test.u32", 7)
    w.add_int32("test.i32", -5)
    w.add_float32("test.f32", 1.5)
    w.add_bool("test.bool", True)
    w.add_string("test.str", "héllo")
    w.add_array("test.arr_i", [1, 2, 3])
    w.add_array("test.arr_s", ["a", "bc"])
    w.add_uint64("test.u64", 1 << 40)
    data = {}
    for name, qt, rows, k in TENSORS:
        if isinstance(qt, str):
            raw = synth.BLOCK_GEN[qt](rng, rows, k)
            w.add_tensor(name, raw, raw_dtype=getattr(gguf.GGMLQuantizationType, qt.upper()))
        else:
            raw = rng.standard_normal((rows, k)).astype(qt)
            if rows == 1:
                raw = raw.reshape(k)
            w.add_tensor(name, raw)
        data[name] = raw
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return data
