"""Writes GWP-0.5 GGUF artifacts from the synthetic weights with the gguf-py
writer, for the loader and artifact-policy tests."""
import numpy as np

SEED = 20261201


def write_artifact(path, g, q8: bool, policy: str | None = None):
    import gguf
    from gguf import quants
    from oracle import synth

    w = synth.make_weights(g, SEED, bias_scale=0.02)
    wr = gguf.GGUFWriter(str(path), "gwp05")
    wr.add_string("gwp05.architecture", "gwp05")
    u32 = {"gwp05.hidden": g.hidden, "gwp05.n_layers": g.layers, "gwp05.n_heads": g.heads,
           "gwp05.head_dim": 128, "gwp05.ffn_dim": g.ffn, "gwp05.action_hidden": g.action_hidden,
           "gwp05.action_ffn_dim": g.action_ffn, "gwp05.action_dim": g.action_dim,
           "gwp05.real_state_dim": g.real_state_dim, "gwp05.real_action_dim": g.real_action_dim,
           "gwp05.num_embodiments": g.num_embodiments, "gwp05.embodiment_id": g.embodiment_id,
           "gwp05.image_height": g.grid_h * 32, "gwp05.image_width": g.grid_w * 32,
           "gwp05.action_chunk": g.action_chunk, "gwp05.inference_steps": g.steps,
           "gwp05.t5_hidden": g.text_dim, "gwp05.vae_z_dim": g.vae_z,
           "gwp05.prompt_tokens": g.prompt_tokens}
    for k, v in u32.items():
        wr.add_uint32(k, v)
    wr.add_float32("gwp05.norm_eps", g.norm_eps)
    if policy:
        from wam_b200.artifact import CONVERTER_REVISION

        wr.add_string("gwp05.weight_policy", policy)
        wr.add_string("gwp05.conversion_policy", policy)
        wr.add_string("gwp05.converter_revision", CONVERTER_REVISION)
    wr.add_float32("gwp05.flow_shift", g.flow_shift)
    for name, bits in w.items():
        inner = synth.linear_inner(name, g)
        if q8 and inner > 0 and inner % 32 == 0:
            f = synth.bf16_bits_to_f32(bits.reshape(-1)).reshape(-1, inner)
            blocks = quants.quantize(f, gguf.GGMLQuantizationType.Q8_0)
            wr.add_tensor(name, blocks, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        else:
            wr.add_tensor(name, bits.reshape(-1, bits.shape[-1]).view(np.uint16),
                          raw_shape=bits.reshape(-1, bits.shape[-1]).shape,
                          raw_dtype=gguf.GGMLQuantizationType.BF16)
    for name, v in synth.statistics(g).items():
        wr.add_tensor(name, v.astype(np.float32))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
