"""CPU model of the expert-parallel peer exchange's signalling (no GPU).

The device side is csrc/ep.cu (ep_pack_kernel / ep_put_kernel ending in signal_peers,
ep_wait_kernel) and the host side duplex/streaming/ep_moe.py (PeerExchange,
ep_forward).  Per layer module and per exchange (dispatch, give-back) every rank owns:
  * one receive buffer with a block per source rank, written by the sources;
  * a flag array with a slot per source rank, and a local epoch counter.
A send writes block `rank` of every destination's buffer, then (the kernel's last CTA)
advances the local epoch and stores it, with release semantics, into slot `rank` of
every destination's flags.  The wait spins (bounded) until every slot of the rank's
own flags has reached the rank's epoch, and the following kernels read the blocks.

Here each rank is a thread that runs these steps in stream order over several layers
and steps, with random delays between the stores (the CTAs of a kernel finish in any
order, ranks drift apart).  The model checks the claim that one buffer per exchange
is enough: every block a rank reads holds exactly the current step's data from its
source, never the previous step's and never the next step's.  A second test shows why
every rank must replay the step graph the same number of times: a rank that runs one
extra step waits on exchanges no peer sends, and its bounded wait gives up.
"""

import random
import threading
import time


class Model:
    def __init__(self, n_ranks, n_layers, seed, wait_limit_s=5.0):
        self.N, self.L = n_ranks, n_layers
        self.rng = random.Random(seed)
        self.lock = threading.Lock()
        # [exchange][layer][dest][source] -> tag (step, source, layer) of the last write
        self.buf = {x: [[[None] * n_ranks for _ in range(n_ranks)] for _ in range(n_layers)]
                    for x in ("disp", "back")}
        self.flags = {x: [[[0] * n_ranks for _ in range(n_ranks)] for _ in range(n_layers)]
                      for x in ("disp", "back")}
        self.epoch = {x: [[0] * n_ranks for _ in range(n_layers)] for x in ("disp", "back")}
        self.violations, self.timeouts = [], []
        self.wait_limit_s = wait_limit_s

    def _jitter(self):
        with self.lock:
            d = self.rng.random()
        time.sleep(d * 2e-4)

    def send(self, x, layer, rank, step):
        """pack / put kernel: the blocks, then the last CTA's epoch store to every peer."""
        dests = list(range(self.N))
        with self.lock:
            self.rng.shuffle(dests)
        for d in dests:                       # CTAs of the grid, in any order
            self._jitter()
            self.buf[x][layer][d][rank] = (step, rank, layer)
        e = self.epoch[x][layer][rank] + 1    # signal_peers: epoch + 1, release stores
        self.epoch[x][layer][rank] = e
        for d in dests:
            self._jitter()
            self.flags[x][layer][d][rank] = e

    def wait(self, x, layer, rank):
        """ep_wait_kernel: every slot of this rank's flags reaches its epoch, bounded."""
        e = self.epoch[x][layer][rank]
        t0 = time.time()
        for s in range(self.N):
            while self.flags[x][layer][rank][s] - e < 0:
                if time.time() - t0 > self.wait_limit_s:
                    self.timeouts.append((x, layer, rank, s))
                    return False
                time.sleep(1e-5)
        return True

    def read(self, x, layer, rank, step):
        """the expert stage (disp) or the rank combine (back) reading every block."""
        for s in range(self.N):
            self._jitter()
            got = self.buf[x][layer][rank][s]
            if got != (step, s, layer):
                self.violations.append((x, layer, rank, s, step, got))

    def rank_steps(self, rank, n_steps):
        for step in range(n_steps):
            for layer in range(self.L):
                self.send("disp", layer, rank, step)      # dispatch pack into the peers
                if not self.wait("disp", layer, rank):
                    return
                self.read("disp", layer, rank, step)      # local experts
                self.send("back", layer, rank, step)      # partials into the owners
                if not self.wait("back", layer, rank):
                    return
                self.read("back", layer, rank, step)      # rank combine


def _run(model, steps_of_rank):
    ts = [threading.Thread(target=model.rank_steps, args=(r, steps_of_rank[r]))
          for r in range(model.N)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=120)
        assert not t.is_alive()


def test_one_buffer_per_exchange_is_never_overwritten_before_it_is_read():
    for n_ranks, seed in ((2, 1), (4, 2), (8, 3)):
        m = Model(n_ranks, n_layers=3, seed=seed)
        _run(m, [6] * n_ranks)
        assert not m.timeouts, m.timeouts[:3]
        assert not m.violations, m.violations[:3]
        # every exchange of every layer ran once per step on every rank
        assert all(e == 6 for x in m.epoch.values() for row in x for e in row)


def test_a_rank_with_one_extra_step_gives_up_instead_of_hanging():
    m = Model(2, n_layers=2, seed=4, wait_limit_s=0.2)
    _run(m, [3, 4])                 # rank 1 replays once more than rank 0
    assert not m.violations
    assert m.timeouts == [("disp", 0, 1, 0)]   # its first wait of the extra step
