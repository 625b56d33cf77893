"""CPU oracle for the speculative-decoding verify path. TEST INFRASTRUCTURE ONLY.

A restatement, in plain torch-on-CPU and numpy, of the reference's algorithm
for the path kvengine's `speculative_greedy` drives (reference files cited per
function). It is the checker the parity tests compare the CUDA path against,
and the CPU baseline `bench.py --impl reference` times. Only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may import it; the
product package (`kvengine_b200`) never does, and has no CPU fallback.

Pinning: the restatement is checked against golden vectors produced by running
the reference itself in the development container (`tests/golden/make_golden.py`
imports kvengine and transformers and writes the fixtures under
`tests/golden/`), see `tests/test_oracle_golden.py`.

Third-party arithmetic restated here: transformers' Qwen2 modules (the
reference does not pin a version; the fixtures were made with transformers
5.5.0 and torch 2.11.0): RMSNorm `w * (x.float() * rsqrt(mean(x^2) + eps)).to(dtype)`,
rotary tables `inv_freq = 1/theta^(2i/hd)`, `cos/sin(pos * inv_freq)` in fp32
cast to the model dtype, rotate-half pairing, SwiGLU `down(silu(gate(x)) * up(x))`,
Linear with bias on q/k/v only, tied lm_head.
"""
