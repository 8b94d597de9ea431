"""The oracle controller on the CPU: statuses, termination, continuity, import
proof, and the host bridge statuses (controller/g4c_b4_resident_epoch.cpp:335-631,
native/resident_epoch_bridge.cpp:424-649; recovery cases of
g4c-attempt70a-r1-*/protocol.md:33-38)."""

import zlib

import numpy as np
import pytest
import torch

from oracle.decoder import OracleDecoder
from oracle.epoch import EpochTrace, OracleEpochController, bridge_execute, compute_slot
from oracle.model import TINY, seeded_weights
from scenario import decode_inputs, import_payload, make_scenario, prefill_epochs


@pytest.fixture(scope="module")
def weights():
    return seeded_weights(TINY, 0)


def controller(weights, dtype=torch.bfloat16):
    return OracleEpochController(OracleDecoder(TINY, weights, dtype))


def prefilled(weights, seed=0, **kw):
    sc = make_scenario(vocab=TINY.vocab, seed=seed, **kw)
    ctl = controller(weights)
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        _, out = ctl.run(**inputs)
        assert out[3] == 0
    return sc, ctl


def test_prefill_writes_prompt_positions_and_resident_state(weights):
    sc, ctl = prefilled(weights)
    for row, prompt in enumerate(sc.prompts):
        if not prompt:
            continue
        assert ctl.res_generation[row] == sc.generations[row]
        assert ctl.res_token[row] == prompt[-1] and ctl.res_position[row] == len(prompt) - 1
        block = int(sc.block_table[row, 0])
        written = ctl.key[:, block, : len(prompt) - 1].float().abs().sum()
        untouched = ctl.key[:, block, len(prompt) - 1:].float().abs().sum()
        assert written > 0 and untouched == 0


@pytest.mark.parametrize("mutate, status", [
    (lambda i: i["control"].__setitem__(0, 9), 201),
    (lambda i: i["control"].__setitem__(0, 0), 201),
    (lambda i: i["control"].__setitem__(5, 1), 205),
    (lambda i: i["control"].__setitem__(6, 1), 206),
    (lambda i: i["control"].__setitem__(1, TINY.vocab), 201),
    (lambda i: i["block_table"].__setitem__(1, i["block_table"][0]), 203),
    (lambda i: i["block_table"].__setitem__(1, 8), 203),
    (lambda i: i["slot"].__setitem__(0, i["slot"][0] + 1), 204),
    (lambda i: i["position"].__setitem__(0, 31) or i["seq_len"].__setitem__(0, 32), 202),
    (lambda i: i["seq_len"].__setitem__(3, 2), 201),
    (lambda i: i["token"].__setitem__(1, -1), 201),
])
def test_recovery_statuses_run_no_step(weights, mutate, status):
    sc, ctl = prefilled(weights, seed=3)
    key0 = ctl.key.clone()
    inputs = decode_inputs(sc, TINY.block_size)
    mutate(inputs)
    history, out = ctl.run(**inputs)
    assert out[3] == status and out[4] == 0
    assert (history == -1).all()
    assert list(out[18:22]) == [3, 3, 3, 3]          # every row finishes with FALLBACK
    assert out[5] == 1                                # fallback flag
    assert torch.equal(key0, ctl.key)


def test_eos_stops_a_row_mid_epoch_and_shrinks_the_batch(weights):
    sc, ctl = prefilled(weights, seed=4)
    probe = controller(weights)
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        probe.run(**inputs)
    inputs = decode_inputs(sc, TINY.block_size)
    inputs["control"][0] = 4
    history, _ = probe.run(**inputs)
    eos = int(history[1, 1])                          # what row 1 emits at step 2
    inputs["control"][1:5] = eos
    history, out = ctl.run(**inputs)
    assert history[1, 1] == eos and (history[2:, 1] == -1).all()
    assert out[6 + 2 * 4 + 1] == 2 and out[6 + 3 * 4 + 1] == 1       # executed 2, reason EOS
    assert out[6 + 4 * 4 + 1] < out[6 + 4 * 4]                         # final active < initial


def test_generation_continuity_is_enforced(weights):
    sc, ctl = prefilled(weights, seed=1)
    inputs = decode_inputs(sc, TINY.block_size)
    _, out = ctl.run(**inputs)
    assert out[3] == 0
    history, out = ctl.run(**inputs)                  # same inputs again: resident state moved on
    assert out[3] == 212


def test_new_generation_clears_the_row_blocks(weights):
    sc, ctl = prefilled(weights, seed=2)
    row = 0
    inputs = decode_inputs(sc, TINY.block_size)
    inputs["token"][row], inputs["position"][row], inputs["seq_len"][row] = 5, 0, 1
    inputs["slot"][row] = compute_slot(TINY, inputs["block_table"], row, 0)
    inputs["control"][3 + 4 + row] = 99               # a new request reuses the row
    _, out = ctl.run(**inputs)
    assert out[3] == 0
    block1 = int(sc.block_table[row, 1])
    assert ctl.key[:, block1].float().abs().sum() == 0


def test_import_checksum_is_the_zlib_adler_of_the_imported_blocks(weights):
    sc, pre = prefilled(weights)
    payload = import_payload(pre.key, pre.value, sc)
    ctl = controller(weights)
    inputs = decode_inputs(sc, TINY.block_size, importing=True)
    _, out = ctl.run(**inputs, import_payload=payload)
    raw = payload.contiguous().view(torch.int16).numpy().tobytes()
    block = TINY.block_size * TINY.kv_width * 2
    expected = 1
    mask = [r for r in range(4) if sc.prompts[r]]
    for cache in range(2):
        for layer in range(TINY.num_layers):
            for row in mask:
                start = ((cache * TINY.num_layers + layer) * 4 + row) * block
                expected = zlib.adler32(raw[start:start + block], expected)
    assert out[3] == 0 and (int(out[5]) & 0xFFFFFFFF) == expected


def test_fp32_mode_runs_the_tiny_configuration(weights):
    sc = make_scenario(vocab=TINY.vocab, seed=0)
    ctl = controller(weights, torch.float32)
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        ctl.run(**inputs)
    trace = EpochTrace()
    history, out = ctl.run(**decode_inputs(sc, TINY.block_size), trace=trace)
    assert out[3] == 0 and out[4] == 2 and trace.logits[0].dtype == torch.float32


@pytest.mark.parametrize("seed", [0, 2, 4])
def test_bf16_epoch_within_tolerance_of_fp32_configuration(weights, seed):
    """Configuration 1 specifies torch fp32; the device computes in bf16.  The
    bf16 restatement of the same epoch stays within the parity rule of the
    fp32 one: tokens equal except at near-ties, logits and KV within 2e-2 per
    vector (measured: about 0.5 % and 0.7 %)."""
    from scenario import check_epoch

    sc = make_scenario(vocab=TINY.vocab, seed=seed)
    bf16, fp32 = controller(weights), controller(weights, torch.float32)
    for inputs in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        bf16.run(**inputs)
        fp32.run(**inputs)
    inputs = decode_inputs(sc, TINY.block_size)
    t16, t32 = EpochTrace(), EpochTrace()
    history, control = bf16.run(**inputs, trace=t16)
    history32, control32 = fp32.run(**inputs, trace=t32)

    class Output:   # the bf16 side in the shape of an engine result
        pass

    out = Output()
    out.history, out.control_out = history, control
    out.logits = np.stack([logits.float().numpy() for logits in t16.logits])
    check = check_epoch(out, history32, control32, t32, inputs, kv=(bf16.key, bf16.value, fp32.key, fp32.value),
                        block_size=TINY.block_size, label=f"bf16 vs fp32 seed {seed}", record=False)
    assert check.logits_err < 1e-2 and check.kv_err < 1e-2


def test_bridge_statuses(weights):
    ctl = controller(weights)
    base = dict(token_ids=[1, 0, 0, 0], positions=[0, 0, 0, 0], seq_lens=[1, 0, 0, 0], eos_ids=[4095] * 4,
                row_generations=[1, 0, 0, 0])
    assert bridge_execute(ctl, 0, 1, configured_eos=4095, **base).ret == 10
    assert bridge_execute(ctl, 1, 9, configured_eos=4095, **base).ret == 10
    assert bridge_execute(ctl, 2, 1, configured_eos=4095, **base).ret == 12
    bad = dict(base, seq_lens=[2, 0, 0, 0])
    assert bridge_execute(ctl, 1, 1, configured_eos=4095, **bad).ret == 11
    ok = bridge_execute(ctl, 1, 2, configured_eos=4095, **base)
    assert ok.ret == 0 and ok.commit_state == 2 and ok.device_status == 0 and ok.executed[0] == 2
    assert ok.declared_input_bytes == 260 and ok.declared_output_bytes == 368


def _poisoned_scenario(weights, seed=6):
    """Seeded cohort (rows 0-2 active) whose row 0 emits, at the first step of a
    K=4 epoch, a token that is in no prompt; returns that token and weights
    whose embedding row for it is NaN."""
    sc, probe = prefilled(weights, seed=seed, active_rows=(1, 1, 1, 0), budget=(8, 8))
    inputs = decode_inputs(sc, TINY.block_size)
    inputs["control"][0] = 4
    history, out = probe.run(**inputs)
    assert out[3] == 0 and out[4] == 4
    poison = int(history[0, 0])
    assert all(poison not in p for p in sc.prompts) and poison not in history[0, 1:3].tolist()
    bad = dict(weights)
    embed = weights["model.embed_tokens.weight"].clone()
    embed[poison] = float("nan")
    bad["model.embed_tokens.weight"] = embed
    return poison, bad, history


def test_non_finite_logits_mid_epoch_fall_back(weights):
    """209 (controller :555-556): the second step's logits of row 0 are NaN.  The
    epoch stops there: the first step's tokens stay in the history, model
    calls = 2, executed = 1 per active row, every row finishes with FALLBACK,
    and the resident state does not advance (:599-614 is not reached)."""
    poison, bad, clean_history = _poisoned_scenario(weights)
    sc, ctl = prefilled(bad, seed=6, active_rows=(1, 1, 1, 0), budget=(8, 8))
    res_position = list(ctl.res_position)
    inputs = decode_inputs(sc, TINY.block_size)
    inputs["control"][0] = 4
    history, out = ctl.run(**inputs)
    assert out[3] == 209 and out[4] == 2
    assert history[0, :3].tolist() == clean_history[0, :3].tolist() and history[0, 0] == poison
    assert (history[1:] == -1).all() and history[0, 3] == -1
    assert list(out[14:18]) == [1, 1, 1, 0]           # executed
    assert list(out[18:22]) == [3, 3, 3, 3]           # every row finishes with FALLBACK
    assert list(ctl.res_position) == res_position


def test_replay_after_a_mid_epoch_fallback_matches_a_clean_run(weights):
    """After a mid-epoch fallback the resident state has not moved (:599-614 is
    not reached), so the same inputs -- same generations -- pass continuity on
    replay; the replay rewrites the KV slots the failed epoch touched and emits
    the tokens of a run that never failed."""
    _, bad, clean_history = _poisoned_scenario(weights)
    sc, ctl = prefilled(bad, seed=6, active_rows=(1, 1, 1, 0), budget=(8, 8))
    inputs = decode_inputs(sc, TINY.block_size)
    inputs["control"][0] = 4
    _, out = ctl.run(**inputs)
    assert out[3] == 209
    ctl.decoder = OracleDecoder(TINY, weights)        # the fault is gone
    history, out = ctl.run(**inputs)
    assert out[3] == 0 and out[4] == 4
    np.testing.assert_array_equal(history, clean_history)


# The reference's epoch case matrix (g4c-attempt69e-r5-*/prepare_inputs.py:12-26):
# K, and per row A(ctive) / E(mpty: never admitted) / F(inished: inactive with
# its length at position + 1).
CASE_MATRIX = [
    ("k1-heterogeneous", 1, "AAAA"),
    ("k2-heterogeneous", 2, "AAAA"),
    ("k4-heterogeneous", 4, "AAAA"),
    ("k8-all-active", 8, "AAAA"),
    ("active-empty-alternating", 4, "AEAE"),
    ("finished-active-empty-active", 4, "FAEA"),
    ("independent-early-eos", 4, "AAAA"),
]


def case_matrix_inputs(weights, name, k, pattern):
    """The seeded cohort of one case and the inputs of its decode epoch (after
    the cohort's prefill epochs)."""
    active_rows = tuple(1 if c == "A" else 0 for c in pattern)
    sc = make_scenario(vocab=TINY.vocab, seed=11, active_rows=active_rows, k=k, budget=(8, 8))
    inputs = decode_inputs(sc, TINY.block_size)
    for r, c in enumerate(pattern):
        if c == "F":
            inputs["token"][r], inputs["position"][r], inputs["seq_len"][r] = 7, 3, 4
            inputs["slot"][r] = compute_slot(TINY, inputs["block_table"], r, 3)
        if c != "A":
            assert inputs["control"][7 + r] == 0
    if name == "independent-early-eos":
        # row r's EOS is the token it emits at step r: the rows stop one after another
        _, probe = prefilled(weights, seed=11, active_rows=active_rows, k=k, budget=(8, 8))
        clean, _ = probe.run(**inputs)
        for r in range(4):
            inputs["control"][1 + r] = int(clean[r, r])
    return sc, inputs


@pytest.mark.parametrize("name, k, pattern", CASE_MATRIX, ids=[c[0] for c in CASE_MATRIX])
def test_epoch_case_matrix(weights, name, k, pattern):
    """Per row: an active row runs until its own EOS or K steps (reason EOS 1 or
    MAX_STEPS 2) and its resident state advances by what it ran; an empty row
    finishes EMPTY (4), a finished row ALREADY_FINISHED (5), and neither
    emits, runs or touches its blocks.  Model calls are the longest row's
    steps; the control output counts the initially and finally active rows."""
    sc, inputs = case_matrix_inputs(weights, name, k, pattern)
    ctl = controller(weights)
    for prefill in prefill_epochs(sc, TINY.block_size, TINY.vocab):
        assert ctl.run(**prefill)[1][3] == 0
    eos = [int(inputs["control"][1 + r]) for r in range(4)]
    key0 = ctl.key.clone()
    history, out = ctl.run(**inputs)
    assert out[3] == 0 and out[0] == k
    executed, reasons = list(out[14:18]), list(out[18:22])
    for r, c in enumerate(pattern):
        column = [int(t) for t in history[:, r]]
        if c != "A":
            assert column == [-1] * 8 and executed[r] == 0 and reasons[r] == (4 if c == "E" else 5)
            for block in sc.block_table[r]:
                assert torch.equal(ctl.key[:, int(block)], key0[:, int(block)])
            continue
        emitted = [t for t in column if t >= 0]
        stop = next((i + 1 for i, t in enumerate(emitted) if t == eos[r]), None)
        assert len(emitted) == executed[r] == (stop or k) and column[executed[r]:] == [-1] * (8 - executed[r])
        assert reasons[r] == (1 if stop else 2)
        assert ctl.res_position[r] == len(sc.prompts[r]) - 1 + executed[r]
        if name == "independent-early-eos":
            assert executed[r] == r + 1
    assert out[4] == max(executed)
    assert out[22] == pattern.count("A") and out[23] == sum(1 for r in range(4) if reasons[r] == 2)


def test_k_step_epoch_equals_k_single_step_epochs(weights):
    """The reference's host-loop route (g4c_b4_epoch_runner.cpp:245-382: one
    decoder call per token, the host feeding each token back) and one resident
    epoch of K steps compute the same thing: tokens, KV cache and resident
    state after K = 4 single-step epochs equal those after one 4-step epoch."""
    sc, resident = prefilled(weights, seed=5, active_rows=(1, 1, 1, 0), budget=(8, 8))
    _, host_loop = prefilled(weights, seed=5, active_rows=(1, 1, 1, 0), budget=(8, 8))
    inputs = decode_inputs(sc, TINY.block_size)
    inputs["control"][0] = 4
    history, out = resident.run(**inputs)
    assert out[3] == 0 and out[4] == 4
    step_inputs = {k: np.array(v, copy=True) for k, v in inputs.items()}
    step_inputs["control"][0] = 1
    tokens = []
    for _ in range(4):
        h, o = host_loop.run(**step_inputs)
        assert o[3] == 0 and o[4] == 1
        tokens.append(h[0].copy())
        for r in range(4):
            if step_inputs["active"][r] and h[0, r] >= 0:
                step_inputs["token"][r] = h[0, r]
                step_inputs["position"][r] += 1
                step_inputs["seq_len"][r] += 1
                step_inputs["slot"][r] = compute_slot(TINY, step_inputs["block_table"], r, int(step_inputs["position"][r]))
    np.testing.assert_array_equal(np.stack(tokens), history[:4])
    assert torch.equal(resident.key, host_loop.key) and torch.equal(resident.value, host_loop.value)
    assert list(resident.res_position) == list(host_loop.res_position)
    assert list(resident.res_token) == list(host_loop.res_token)
