"""The peer-memory all-gather's slot/epoch protocol (retree_b200.peer), model-checked on the CPU.

Each rank runs, per layer, the steps the fused forward issues on its stream:
its attention writes slot ``layer % 2`` of its own buffer, ``signal`` stores
the layer's epoch into its entry of every rank's flag array, and ``gather``
waits for each source's flag and then reads that source's slot.  A random
scheduler interleaves the ranks step by step (a gather's wait and its read of
each source are separate steps); every read must see the data of the layer it
waited for.  With an odd layer count two consecutive layers share a slot
across the forward boundary, and the model finds the overwrite the forward
refuses to risk (``FusedTarget`` requires an even count).
"""

import random


def _run(world: int, layers: int, forwards: int, seed: int) -> bool:
    rng = random.Random(seed)
    slots = [[None, None] for _ in range(world)]       # slots[rank][s] = (epoch, rank) written there
    flags = [[0] * world for _ in range(world)]        # flags[reader][src]
    # per rank: a program of steps, generated lazily from (epoch index, phase, source)
    steps = []
    for r in range(world):
        prog = []
        for k in range(forwards * layers):
            layer = k % layers
            epoch = k + 1
            prog.append(("write", layer % 2, epoch))
            prog.append(("signal", epoch))
            for src in rng.sample(range(world), world):   # a gather's CTAs run in any order
                prog.append(("wait", src, epoch))
                prog.append(("read", src, layer % 2, epoch))
        steps.append(prog)
    pc = [0] * world
    ok = True
    while any(pc[r] < len(steps[r]) for r in range(world)):
        runnable = []
        for r in range(world):
            if pc[r] >= len(steps[r]):
                continue
            op = steps[r][pc[r]]
            if op[0] == "wait" and flags[r][op[1]] < op[2]:
                continue
            runnable.append(r)
        assert runnable, "deadlock"
        r = rng.choice(runnable)
        op = steps[r][pc[r]]
        pc[r] += 1
        if op[0] == "write":
            slots[r][op[1]] = (op[2], r)
        elif op[0] == "signal":
            for p in range(world):
                flags[p][r] = max(flags[p][r], op[1])
        elif op[0] == "read":
            _, src, s, epoch = op
            if slots[src][s] != (epoch, src):
                ok = False
    return ok


def test_two_slots_by_layer_parity_never_expose_the_wrong_layer():
    for world in (2, 3, 4, 8):
        for seed in range(150):
            assert _run(world, layers=4, forwards=3, seed=seed), (world, seed)


def test_an_odd_layer_count_can_overwrite_a_slot_still_being_read():
    # the same protocol with 3 layers: layer 2 and the next forward's layer 0 share slot 0
    assert not all(_run(2, layers=3, forwards=3, seed=s) for s in range(400))
