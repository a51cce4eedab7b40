"""CPU oracle for the slot_murmurate hot path.

TEST INFRASTRUCTURE ONLY. This package is a CPU restatement of the reference
implementation (beaglabs/murmurative-attention, src/murmurative/reference.py)
used as the checker for the CUDA path. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs may import it. The product path
(murmurative_attention_b200) never imports or falls back to it.

Parity pin: tests/golden/*.npz were produced by tests/golden/make_golden.py,
which imports the real reference.py in the build container and runs it on
seeded inputs; tests/test_oracle_golden.py checks this restatement against
those fixtures.
"""

from .murmurate import (  # noqa: F401
    slot_select,
    slot_attend,
    slot_update,
    slot_diffusion,
    slot_murmurate,
    slot_murmurate_forced,
    slot_murmurate_trace,
    slot_murmurate_backward_explicit,
    slot_murmurate_layer_reference,
    make_inputs,
    row_gap_ok,
)
