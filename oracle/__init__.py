"""CPU oracle for the Breeze-TTS-2 streaming-decode hot path.

TEST INFRASTRUCTURE ONLY.  This package restates, in numpy and plain C, the arithmetic of the reference's
decode path (the official eager PyTorch modules that AsherHou/Breeze-TTS-2-flash accelerates).  It is imported
only by ``tests/``, by ``__graft_entry__.smoke()`` as the checker, and by ``bench.py``'s CPU-baseline leg and
``--impl reference`` arm.  The product path (``breeze-tts-2-flash_b200/flashb``) never imports it and has no CPU
fallback: without the CUDA library it raises.

Every function cites the reference file:line it follows.  Citations are relative to the reference project root;
``UP/`` abbreviates ``third_party/breeze-tts/`` (the vendored official runtime).

Parity pins: ``tests/golden/make_golden.py`` imports the reference's own PyTorch modules (official
``DepthDecoderGraph``, ``BackboneGraph`` with Qwen3 layers, ``eager_attention_forward``, ``BreezeRMSNorm``) in the
build container and records their outputs on seeded inputs as ``tests/golden/*.npz``; ``tests/test_oracle_golden.py``
checks this oracle against those fixtures.

Modules
  bf16     bf16 round-to-nearest-even emulation on float32 arrays
  decode   RMSNorm, linear, RoPE, GQA decode attention, Qwen3 backbone layer/step, lm_head, CFG
  depth    depth-decoder frame (16 codebook steps, eager rounding points) using ``sampler``
  sampler  ctypes wrapper of sampler.c: the bit-exact CFG/top-k/top-p/argmax(p/q) sampler and exp routine
  prefill  causal GQA prefill attention (eager semantics)
"""
