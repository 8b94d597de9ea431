"""CPU oracle for the resident decode epoch -- TEST INFRASTRUCTURE ONLY.

Nothing in the product (``cruise_b200``) imports, links or executes anything
under this directory.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and there
only as the checker or as the timed CPU baseline.

Contents
--------
``synth``    seeded weight generator (splitmix64 -> Irwin-Hall(4) -> bf16),
             the CPU restatement of the generator the engine runs on the GPU.
``decoder``  the Qwen2 paged decoder step, restating
             ``history/attempts/g4c-attempt69c-b4-air/batched_decoder_step.py:197-417``
             with the CPU bodies of its custom ops
             (``g4a_linear_t.py:17-18``, ``g4a_linear_t_bias.py:18-21``,
             ``qk-attempt50/export_qk_attempt50_air.py:47-56``; the
             barrier/materialize ops are identities, ``bf16_barrier.cpp:47-50``).
``epoch``    the device epoch controller ``controller/g4c_b4_resident_epoch.cpp:177-631``
             and the host bridge ``native/resident_epoch_bridge.cpp:424-649``.

Parity pin: ``tests/golden/make_golden.py`` imports the reference's own
``PagedQwenDecoderStep`` (geometry constants patched in, the documented CPU op
bodies registered) and records its outputs.  The geometries are tiny and a
1-layer shape with the 7B model's attention (7 query heads per KV head, head
size 128).  ``tests/test_oracle_golden.py`` checks this oracle bit-exactly
against those fixtures.
"""
