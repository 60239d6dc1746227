"""CPU: the reference's own STD decode on the reduced random-init decoder
(tests/golden/acceptance_reduced.npz, written by make_acceptance.py from the
reference's std_generate_qwen25vl / ar_generate_qwen25vl on CPU, fp16):
token-exact to its AR decode, and it accepts almost nothing -- at configs[4]'s
selected-to-visual ratio random weights leave the sparse draft and the dense
model disagreeing on nearly every token."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_reference_acceptance_on_random_weights_is_near_zero():
    g = np.load(os.path.join(GOLDEN, "acceptance_reduced.npz"))
    acc = g["accept_lengths"]
    assert np.array_equal(g["std_tokens"], g["ar_tokens"])
    for row in acc:
        a = row[row >= 0]
        assert len(a) >= 20
        assert a.sum() / (9 * len(a)) < 0.05
    assert int(g["threads"]) >= 1 and float(g["std_decoding_s"].sum()) > 0
