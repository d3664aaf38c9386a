"""CPU oracle for the qwenedit_b200 hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs may import
this package, and only to check results or as the timed CPU baseline. Nothing in ``qwenedit_b200`` imports it.

Contents
* ``latents_ref`` — the reference's per-step latent ops in torch eager (MaskState.blend, _compose, the
  stored_latents crop), pinned to golden outputs of the reference's own code (tests/golden/latents.npz).
* ``radix_ref``  — restatement of SGLang's RadixCache + TokenToKVPoolAllocator as QwenEdit's PagedKVPool
  drives them (multi_turn/cache/paged.py:52-131). SGLang (pinned at e6072935b by scripts/setup.sh:11-14) is
  not vendored; its behaviour is restated from the call sites and from the published RadixCache design.
  **Slot assignment and eviction order: parity unpinned** against real SGLang (no reference test fixes
  them); the reference's own tests (tests/test_paged.py:28-65) are replayed against it.
* ``pool_ref``   — the reference PagedKVPool on CPU: ``index_select`` / ``index_copy_`` data movement
  (paged.py:106-116) over ``radix_ref``.
* ``nvfp4_ref.c`` / ``nvfp4_ref`` — C restatement of the Triton NVFP4 kernels (multi_turn/fibo/fp4.py:37-91)
  with GPU roundings; pinned against the reference kernels run under Triton's interpreter
  (tests/golden/gen_golden.py).
"""
