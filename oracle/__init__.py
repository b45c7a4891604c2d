"""CPU oracle of the ZONOS3-Mini hot path — TEST INFRASTRUCTURE, never product code.

A restatement in plain PyTorch (CPU, float32 unless a function says otherwise) of the reference's own
implementation of the three hot-path parts, each function citing the reference file:line it follows:

* ``oracle.gdn``     — gated DeltaNet layer and recurrence (model/src/zonos3/reference/lm.py:556-602)
* ``oracle.attnres`` — Full AttnRes route (lm.py:384-389; servers/sgl/.../models/zonos3.py:99-113 and the Triton
  kernel's rounding points, servers/sgl/.../models/training_attnres_kernels.py:1268-1348)
* ``oracle.moe``     — router, top-k, permutation and SwiGLU experts (lm.py:604-639; zonos3.py:746-828;
  layers/moe/fused_moe/layer.py:159-161)
* ``oracle.sampler`` — the TTS sampler's masks, penalty and filters (model/src/zonos3/tts/sampler.py:59-372)
* ``oracle.attention`` — decode attention over a slot-indexed KV cache and the KV store (lm.py:526-531;
  servers/sgl/.../attention/fa.py:64-81; servers/sgl/.../kernel/csrc/jit/store.cu:28-50)

The restatement is pinned against golden vectors produced by the unmodified reference (``tests/golden/``).
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may import this
package, and only as the checker or the timed CPU baseline; the CUDA path never calls it.
"""
