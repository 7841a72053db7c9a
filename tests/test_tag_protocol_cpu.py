"""The one-bit layer tag of the persistent decode step's partial sums (csrc/decode_mk.cu), checked
as a protocol on the CPU: CTAs (on one or several ranks) each own one o slot and one down slot;
per layer a CTA waits until every o slot shows the layer's parity, writes its down slot, waits
until every down slot shows it, then writes its o slot for the next layer. Any interleaving the
waits allow is explored at random; a reader must never accept a value from another layer or step.
(The ATTN / WGU steps in between are local to a CTA here; the real kernel's local barriers only
remove interleavings.)"""

import random


def _run(n_ctas, n_layers, n_steps, seed):
    rng = random.Random(seed)
    # slot value = (step, layer) of its last write; the tag bit is (step * L + layer) & 1
    init = (-1, n_layers - 1)  # the buffers start with the parity layer 0 of step 0 does not expect
    o_slot = [init] * n_ctas
    d_slot = [init] * n_ctas
    tag = lambda v: (v[0] * n_layers + v[1]) & 1  # noqa: E731
    # per CTA program counter: (step, layer, phase); phase 0: write o(l) [needs down(l-1) all seen],
    # phase 1: write down(l) [needs o(l) all seen]
    pc = [(0, 0, 0)] * n_ctas
    done = 0
    while done < n_ctas:
        ready = []
        for c in range(n_ctas):
            s, l, ph = pc[c]
            if s == n_steps:
                continue
            if ph == 0:
                need, slots = ((s, l - 1) if l else (s - 1, n_layers - 1)), d_slot
            else:
                need, slots = (s, l), o_slot
            first = (s, l, ph) == (0, 0, 0)  # layer 0 of the first step reads the embedding instead
            want = tag(need) if need[0] >= 0 else None
            ok = first or all(tag(v) == want for v in slots)
            if ok:
                if not first:
                    for v in slots:  # what the tag accepted must be exactly the expected write
                        assert v == need, (c, pc[c], v, need)
                ready.append(c)
        assert ready, "deadlock"
        c = rng.choice(ready)
        s, l, ph = pc[c]
        if ph == 0:
            o_slot[c] = (s, l)
            pc[c] = (s, l, 1)
        else:
            d_slot[c] = (s, l)
            nl = l + 1
            pc[c] = (s, nl, 0) if nl < n_layers else (s + 1, 0, 0)
            if pc[c][0] == n_steps:
                done += 1


def test_one_bit_tag_never_accepts_a_stale_value():
    for seed in range(200):
        _run(n_ctas=random.Random(seed).randint(2, 6), n_layers=random.Random(seed + 1).randint(1, 5),
             n_steps=3, seed=seed)
