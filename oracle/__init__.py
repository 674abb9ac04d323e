"""CPU oracle for the strands-decider scoring prefill.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this package.
Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py`
use it, and only as the checker or as the timed CPU baseline, never as the thing
measured or shipped.

Contents:
  quant.py  - bit-exact numpy restatement of the packed weight formats (int4
              group-128, NVFP4, ternary) and of their dequantisation. The
              reference ships no quantiser, so these functions are the single
              source of truth for the dequantised weights.
  torso.py  - torch fp32 restatement of the Qwen3.5 hybrid torso the reference
              runs (transformers 5.5 `models/qwen3_5/modeling_qwen3_5.py`,
              cited as `TF:line`), with ragged sequences and an explicit
              prefix cache (GDN recurrent state, conv history, attention KV).
  head.py   - the option-token decision head and the answer read-back math
              (`src/strands_decider/modeling.py`, `schema.py`, `infer.py`).
  synth.py  - the seeded synthetic workloads used by the parity tests.

Pinning: `tests/golden/make_golden.py` runs the reference itself (transformers'
Qwen3_5TextModel plus strands_decider's own readout functions) in the build
container and commits the outputs as fixtures; `tests/test_oracle_pins.py`
checks this oracle against them.
"""
