"""Host-side sizing logic of the model forward (no GPU)."""
import types

from neuratensor_b200 import NeuraTensorModel, get_preset


def _groups(preset, seq):
    fake = types.SimpleNamespace(config=get_preset(preset), MAX_ACTIVATION_ELEMS=NeuraTensorModel.MAX_ACTIVATION_ELEMS)
    return NeuraTensorModel.group_size(fake, seq)


def test_sequence_groups_keep_activations_under_the_limit():
    # large preset: in_proj output is 2*4096 wide, so 16 streams of 8192 per pass
    assert _groups("large", 8192) == 16
    # the small-preset prefill (8 x 2048) runs in one pass
    assert _groups("small", 2048) >= 8
    # a single token step never groups
    assert _groups("large", 1) >= 64
    for preset in ("pico", "small", "medium", "large"):
        c = get_preset(preset)
        width = max(2 * c.d_model * c.expand, 3 * c.d_model)
        for seq in (1, 100, c.max_seq_len):
            g = _groups(preset, seq)
            assert g >= 1 and g * seq * width <= NeuraTensorModel.MAX_ACTIVATION_ELEMS
