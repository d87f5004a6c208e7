"""GGUF layer loading on the CPU side (gx_gguf_inspect_layer needs no device): the layer's
shapes, types and rotation from a file written like the reference model file, and the header
checks of src/gguf.zig:263-334 on malformed files."""
import numpy as np
import pytest

from gyro_moe import abi, synth
import gguf_file


def small_layers(shared: bool = True):
    layers = [synth.make_layer(70 + i, n_expert=8, E=256, F=128, U=2, expert_weights_scale=2.5) for i in range(2)]
    for l in layers[1:]:                      # one sign vector per width for the whole file
        l["gate_signs"], l["down_signs"] = layers[0]["gate_signs"], layers[0]["down_signs"]
    if shared:
        layers[1]["shared"] = synth.make_shared(80, E=256, SF=128, type_id=abi.GX_Q8_0)
    return layers


def test_inspect_reports_the_layer(tmp_path):
    path = tmp_path / "m.gguf"
    gguf_file.model_file(path, small_layers())
    for i, shared in ((0, False), (1, True)):
        info = abi.gguf_layer_info(path, i)
        assert (info.type_id, info.n_expert, info.n_embd, info.n_ff, info.n_used) == (144, 8, 256, 128, 2)
        assert info.expert_weights_scale == pytest.approx(2.5)
        assert info.rotated == 3
        if shared:
            assert (info.shared_type, info.shared_ff) == (abi.GX_Q8_0, 128)
        else:
            assert info.shared_type == abi.GX_SHARED_NONE


def test_identity_sign_mode_and_unrotated_layers(tmp_path):
    layers = [synth.make_layer(90, n_expert=8, E=256, F=128, U=2, signs=False)]
    gguf_file.model_file(tmp_path / "plain.gguf", layers)
    assert abi.gguf_layer_info(tmp_path / "plain.gguf", 0).rotated == 0


def expect(code, path, layer=0):
    with pytest.raises(abi.GxError) as e:
        abi.gguf_layer_info(path, layer)
    assert e.value.code == code


def test_malformed_files_are_refused(tmp_path):
    layers = small_layers(shared=False)
    good = tmp_path / "good.gguf"
    gguf_file.model_file(good, layers)
    data = good.read_bytes()
    (tmp_path / "magic.gguf").write_bytes(b"GGUX" + data[4:])
    expect(-1, tmp_path / "magic.gguf")
    (tmp_path / "short.gguf").write_bytes(data[:200])
    expect(-1, tmp_path / "short.gguf")
    gguf_file.model_file(tmp_path / "v2.gguf", layers, version=2)
    expect(-5, tmp_path / "v2.gguf")
    gguf_file.model_file(tmp_path / "misaligned.gguf", layers, misalign="blk.0.ffn_up_exps.weight")
    expect(-1, tmp_path / "misaligned.gguf")
    gguf_file.model_file(tmp_path / "overlap.gguf", layers, overlap=(0, 1))
    expect(-1, tmp_path / "overlap.gguf")
    expect(-1, tmp_path / "absent.gguf")
    expect(-1, good, layer=5)                 # no such layer
    gguf_file.model_file(tmp_path / "mode.gguf", layers, sign_mode="implicit")
    expect(-5, tmp_path / "mode.gguf")


def test_gate_and_up_must_share_signs(tmp_path):
    layers = small_layers(shared=False)
    tensors, rotated = gguf_file.layer_records(0, layers[0])
    l0 = layers[0]
    flipped = [int(v) for v in -l0["gate_signs"]]
    meta = [("general.architecture", gguf_file.STR, "qwen4exp"), ("qwen4exp.expert_used_count", gguf_file.U32, 2),
            ("prism.hadamard.version", gguf_file.U32, 1), ("prism.hadamard.block_size", gguf_file.U32, 128),
            ("prism.hadamard.transform", gguf_file.STR, "normalized-sylvester-walsh-hadamard"),
            ("prism.hadamard.axis", gguf_file.STR, "input-last-dimension"),
            ("prism.hadamard.sign_mode", gguf_file.STR, "explicit"),
            # the up tensor is listed, the gate tensor is not: their inputs would differ
            ("prism.hadamard.weight_names", gguf_file.ARR, (gguf_file.STR, ["blk.0.ffn_up_exps.weight"])),
            ("prism.hadamard.sign_widths", gguf_file.ARR, (gguf_file.I32, [256])),
            ("prism.hadamard.sign_values", gguf_file.ARR, (gguf_file.I32, flipped))]
    gguf_file.write(tmp_path / "signs.gguf", meta, tensors)
    expect(-1, tmp_path / "signs.gguf")
