"""The CPU rollout's stochastic update masks (run_rollout_from_particles,
crates/burn_automata/src/rollout/mod.rs:222-238, stochastic_mask :644-651).

The reference draws them from rand 0.9.4's StdRng (rand_chacha 0.9.0
ChaCha12Rng seeded by rand_core 0.9's seed_from_u64).  No Rust toolchain and
no golden values exist here, so the seeding and the 12-round stream are
unpinned; what is pinned:
  CPU: the oracle's ChaCha block function at 20 rounds against OpenSSL's
       ChaCha20 keystream (the `cryptography` package), and the oracle's
       seeding, word positions and float draw against an independent
       pure-Python restatement;
  GPU: the device masks against the oracle bit for bit, and GPU rollouts with
       update_prob < 1 against the oracle rollout fed the oracle's masks."""

import numpy as np
import pytest

import oracle
from burn_automata_b200 import workloads

M32 = 0xFFFFFFFF
M64 = 0xFFFFFFFFFFFFFFFF


def py_seed_from_u64(state):
    """PCG32 (XSH-RR 64/32) seed expansion, restated independently."""
    key = []
    for _ in range(8):
        state = (state * 6364136223846793005 + 11634580027462260723) & M64
        xorshifted = (((state >> 18) ^ state) >> 27) & M32
        rot = state >> 59
        key.append(((xorshifted >> rot) | (xorshifted << ((32 - rot) % 32))) & M32)
    return np.array(key, np.uint32)


def py_chacha_block(key, counter, rounds):
    def rotl(v, r):
        return ((v << r) | (v >> (32 - r))) & M32

    state = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574] + [int(k) for k in key] + [
        counter & M32, counter >> 32, 0, 0]
    x = list(state)

    def qr(a, b, c, d):
        x[a] = (x[a] + x[b]) & M32
        x[d] = rotl(x[d] ^ x[a], 16)
        x[c] = (x[c] + x[d]) & M32
        x[b] = rotl(x[b] ^ x[c], 12)
        x[a] = (x[a] + x[b]) & M32
        x[d] = rotl(x[d] ^ x[a], 8)
        x[c] = (x[c] + x[d]) & M32
        x[b] = rotl(x[b] ^ x[c], 7)

    for _ in range(rounds // 2):
        qr(0, 4, 8, 12)
        qr(1, 5, 9, 13)
        qr(2, 6, 10, 14)
        qr(3, 7, 11, 15)
        qr(0, 5, 10, 15)
        qr(1, 6, 11, 12)
        qr(2, 7, 8, 13)
        qr(3, 4, 9, 14)
    return np.array([(a + b) & M32 for a, b in zip(x, state)], np.uint32)


@pytest.mark.parametrize("counter", [0, 1, 7, 123456])
def test_chacha20_block_matches_openssl(counter):
    Cipher = pytest.importorskip("cryptography.hazmat.primitives.ciphers")
    rng = np.random.default_rng(counter + 3)
    key = rng.integers(0, 2**32, 8, dtype=np.uint64).astype(np.uint32)
    # OpenSSL's 16-byte ChaCha20 IV: 32-bit little-endian block counter, then
    # the 96-bit nonce (0): the same state as a 64-bit counter with stream 0.
    iv = int(counter).to_bytes(4, "little") + bytes(12)
    enc = Cipher.Cipher(Cipher.algorithms.ChaCha20(key.tobytes(), iv), mode=None).encryptor()
    want = np.frombuffer(enc.update(bytes(128)), dtype="<u4")
    got = np.concatenate([oracle.chacha_block(key, counter + b, 20) for b in range(2)])
    np.testing.assert_array_equal(got, want)


def test_chacha12_and_seeding_match_a_python_restatement():
    for seed in (0, 42 ^ 0x5EED, 2**63 + 5, M64):
        np.testing.assert_array_equal(oracle.stdrng_key(seed), py_seed_from_u64(seed))
    key = py_seed_from_u64(7)
    for counter in (0, 3, 2**32 - 1, 2**32 + 9):
        np.testing.assert_array_equal(oracle.chacha_block(key, counter, 12),
                                      py_chacha_block(key, counter, 12))


def test_masks_follow_the_stream_word_by_word():
    seed, p, count = 42, 0.5, 37  # 37 words per step: blocks straddle the steps
    key = py_seed_from_u64(seed ^ 0x5EED)
    masks = oracle.rollout_masks(seed, p, count, 3)
    words = np.concatenate([py_chacha_block(key, b, 12) for b in range(8)])
    u = (words[:3 * count] >> 8).astype(np.float32) * np.float32(1.0 / 16777216.0)
    np.testing.assert_array_equal(masks.reshape(-1), (u < np.float32(p)).astype(np.float32))
    np.testing.assert_array_equal(oracle.rollout_masks(seed, p, count, 1, first_step=2)[0],
                                  masks[2])


def test_mask_edges_and_rate():
    assert np.all(oracle.rollout_masks(1, 1.0, 100, 2) == 1.0)
    assert np.all(oracle.rollout_masks(1, 0.0, 100, 2) == 0.0)
    m = oracle.rollout_masks(9, 0.3, 20000, 2)
    assert abs(float(m.mean()) - 0.3) < 0.01
    assert not np.array_equal(m[0], m[1])


@pytest.mark.gpu
@pytest.mark.parametrize("seed,p,count,first,steps", [(42, 0.5, 4096, 0, 3), (7, 0.25, 1000, 5, 2),
                                                      (2**64 - 1, 0.9, 4097, 3, 2),
                                                      (3, 0.5, 1 << 20, 1, 1)])
def test_gpu_masks_match_the_oracle(seed, p, count, first, steps):
    import burn_automata_b200 as ba

    got = ba.rollout_update_masks(seed, p, count, steps, first_step=first)
    want = oracle.rollout_masks(seed, p, count, steps, first_step=first)
    np.testing.assert_array_equal(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("log_norm,batch", [(False, 1), (True, 1), (False, 3)])
def test_gpu_stochastic_rollout_matches_the_oracle(oracle_mod, log_norm, batch):
    """One mask stream over the whole batch (stochastic_mask draws
    batch * particle_count values per step)."""
    import burn_automata_b200 as ba

    w = workloads.make("cfg0", n=2048, batch=batch)
    w.model = w.model.with_(log_norm_grad=log_norm)
    m = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                           w.weights.b2))
    steps, p, seed = 12, 0.5, 42
    cfg = ba.RolloutConfig(batch_size=batch, particle_count=w.n, steps=steps, dt=w.dt,
                           update_prob=p, seed=seed)
    trace = ba.run_rollout_from_particles(m, w.grid, cfg, w.positions, w.states)
    masks = oracle_mod.rollout_masks(seed, p, batch * w.n, steps)
    pos, st, mean_dx = oracle_mod.rollout(w.model, w.weights, w.grid, w.positions, w.states,
                                          batch, w.n, steps, w.dt, masks=masks)
    if log_norm:
        # the rollout tolerance: log1p is correctly rounded on the GPU, the
        # host's log1pf is not, and the rare one-ulp differences grow over steps
        for a, b in ((trace.states, st), (trace.positions, pos)):
            assert np.linalg.norm(a.astype(np.float64) - b) <= 1e-3 * np.linalg.norm(b)
    else:
        np.testing.assert_array_equal(trace.states, st)
        np.testing.assert_array_equal(trace.positions, pos)
    np.testing.assert_allclose(trace.mean_dx, mean_dx, rtol=1e-5)
    # the unmasked rollout differs: the mask was applied
    full = ba.run_rollout_from_particles(
        m, w.grid, ba.RolloutConfig(batch_size=batch, particle_count=w.n, steps=steps, dt=w.dt),
        w.positions, w.states)
    assert not np.array_equal(full.states, trace.states)
    m.close()
