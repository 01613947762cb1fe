"""Model of the barrier protocol of one head of the triangle-attention core (k_triatt_core_tc in
sparsefold_b200/csrc/sf_triatt_tc.cu), run under many random interleavings on the CPU.

Actors: the head's issue thread, its four softmax warps, the tensor core (MMAs run one at a
time in issue order; a commit arrives once everything issued before it has run) and the TMA
engine (loads land in any order, at any later time).  Every mbarrier is a phase counter, and
every parity wait checks, each time it polls, that the barrier has completed either exactly
the phases before the one waited for or one more: `mbarrier.try_wait.parity` cannot tell
phases further apart, so any other state would be a wait that passes too early or never.
Ring slots and TMEM buffers carry the block they hold, and every reader checks it sees the
block it expects, so a refill that overwrites data still in use is caught.
"""
import random

import pytest

RING, VRING = 4, 6


class Bar:
  def __init__(self, name, count):
    self.name, self.count, self.arrived, self.done = name, count, 0, 0

  def arrive(self):
    self.arrived += 1
    assert self.arrived <= self.count, f"{self.name}: too many arrivals"
    if self.arrived == self.count:
      self.arrived, self.done = 0, self.done + 1

  def ready(self, use):
    # what the hardware can distinguish: `use` (not yet) or `use + 1` (done)
    assert self.done in (use, use + 1), f"{self.name}: waiting for use {use} with {self.done} phases complete"
    return self.done == use + 1


class Head:
  def __init__(self, nkb, rng, rescale_p, early_pready=False):
    # early_pready plants a mistake in the model (P_j signalled before it is written), to show
    # that the model catches it
    self.nkb, self.rng, self.rescale_p, self.early_pready = nkb, rng, rescale_p, early_pready
    self.sbar = [Bar(f"sbar{i}", 2) for i in range(2)]
    self.pvbar = [Bar(f"pvbar{i}", 1) for i in range(2)]
    self.pready = [Bar(f"pready{i}", 4) for i in range(2)]
    self.lbar = [Bar(f"lbar{i}", 2) for i in range(RING)]    # expect_tx arrival + the bytes landing
    self.rbar, self.wbar = Bar("rbar", 2), Bar("wbar", 2)
    self.kslot = [None] * RING
    self.bslot = [None] * RING
    self.vslot = [None] * VRING
    self.tmem = [None, None]       # S buffers: ("S", j) or ("P", j)
    self.mma = []                  # issued, not yet run: (kind, arg)
    self.tma = []                  # in flight: (slot list, index, value, barrier)
    self.s_read = [0] * 4          # per softmax warp: blocks whose S it has read
    self.p_written = {}            # block -> warps that wrote their P rows

  # ---- issue thread ----
  def load(self, jj):
    bar = self.lbar[jj % RING]
    bar.arrive()   # expect_tx
    for slots, idx in ((self.kslot, jj % RING), (self.bslot, jj % RING), (self.vslot, jj % VRING)):
      slots[idx] = ("loading", jj)
      self.tma.append((slots, idx, jj, bar))

  def issuer(self):
    nkb = self.nkb
    self.load(0)
    self.load(1)
    yield None   # Q reaches TMEM (CTA barrier)

    def issue_s(jj):
      while not self.lbar[jj % RING].ready(jj // RING):
        yield ("lbar", jj)
      self.sbar[jj & 1].arrive()
      self.mma.append(("S", jj))
      self.mma.append(("commit", self.sbar[jj & 1]))
      yield None

    yield from issue_s(0)
    self.load(2)
    yield None
    yield from issue_s(1)
    self.load(3)
    yield None
    for j in range(nkb):
      while not self.pready[j & 1].ready(j >> 1):
        yield ("pready", j)
      self.mma.append(("PV", j))
      self.mma.append(("commit", self.pvbar[j & 1]))
      yield None
      if j + 2 < nkb:
        yield from issue_s(j + 2)
      if j + RING < nkb:
        self.load(j + RING)
      elif j + RING == nkb:          # residual into the bias slot of block nkb-4
        self.rbar.arrive()
        self.bslot[nkb % RING] = ("loading", "resid")
        self.tma.append((self.bslot, nkb % RING, "resid", self.rbar))
      elif j + RING == nkb + 1:      # W_o into the bias slot of block nkb-3
        self.wbar.arrive()
        self.bslot[(nkb + 1) % RING] = ("loading", "wo")
        self.tma.append((self.bslot, (nkb + 1) % RING, "wo", self.wbar))
      yield None

  # ---- a softmax warp ----
  def softmax(self, w):
    nkb = self.nkb
    for j in range(nkb):
      while not self.sbar[j & 1].ready(j >> 1):
        yield ("sbar", j)
      if self.early_pready:
        self.pready[j & 1].arrive()
      elif j >= 1:
        self.pready[(j - 1) & 1].arrive()   # P_{j-1}, stored at the end of the previous block
      assert self.tmem[j & 1] == ("S", j), f"softmax {w} block {j} reads {self.tmem[j & 1]}"
      assert self.bslot[j % RING] == j, f"softmax {w} block {j} bias slot holds {self.bslot[j % RING]}"
      self.s_read[w] += 1
      yield None
      # (every state change above is followed by a yield of None, so the scheduler sees progress)
      if j >= 1 and self.rng.random() < self.rescale_p:   # the running max moved: rescale O
        while not self.pvbar[(j - 1) & 1].ready((j - 1) >> 1):
          yield ("pvbar", j - 1)
      assert self.tmem[j & 1] in (("S", j), ("P", j)), f"softmax {w} writes P_{j} over {self.tmem[j & 1]}"
      self.p_written.setdefault(j, set()).add(w)
      if len(self.p_written[j]) == 4:
        self.tmem[j & 1] = ("P", j)
      yield None
    if not self.early_pready:
      self.pready[(nkb - 1) & 1].arrive()
    yield None
    for jj in (nkb - 2, nkb - 1):
      while not self.pvbar[jj & 1].ready(jj >> 1):
        yield ("pvbar-end", jj)
    # gated O staged in the bias slot of block nkb-1; the residual and W_o must have landed
    slot = (nkb - 1) % RING
    assert not any(s is self.bslot and i == slot for s, i, _, _ in self.tma), "ostage slot still being loaded"
    self.bslot[slot] = "ostage"
    yield None
    while not self.rbar.ready(0) or not self.wbar.ready(0):
      yield ("epilogue", None)
    assert self.bslot[nkb % RING] == "resid" and self.bslot[(nkb + 1) % RING] == "wo"

  # ---- tensor core and TMA engine: one step each ----
  def run_mma(self):
    kind, arg = self.mma.pop(0)
    if kind == "S":
      assert self.kslot[arg % RING] == arg, f"S_{arg} reads K slot {self.kslot[arg % RING]}"
      prev = self.tmem[arg & 1]
      assert prev is None or prev == ("P", arg - 2), f"S_{arg} overwrites {prev}"
      self.tmem[arg & 1] = ("S", arg)
    elif kind == "PV":
      assert self.tmem[arg & 1] == ("P", arg), f"PV_{arg} reads {self.tmem[arg & 1]}"
      assert self.vslot[arg % VRING] == arg, f"PV_{arg} reads V slot {self.vslot[arg % VRING]}"
    else:
      arg.arrive()

  def land(self):
    slots, idx, val, bar = self.tma.pop(self.rng.randrange(len(self.tma)))
    slots[idx] = val
    if not any(b is bar for _, _, _, b in self.tma):   # all bytes of this barrier's loads are in
      bar.arrive()


def simulate(nkb, seed, rescale_p, early_pready=False):
  rng = random.Random(seed)
  h = Head(nkb, rng, rescale_p, early_pready)
  actors = {a: g for a, g in enumerate([h.issuer()] + [h.softmax(w) for w in range(4)])}

  def step(a):
    """Advance actor a once; True if it made progress (not blocked on a wait)."""
    try:
      return next(actors[a]) is None
    except StopIteration:
      del actors[a]
      return True

  for _ in range(400000):
    if not actors and not h.mma and not h.tma:
      break
    choices = list(actors) + (["mma"] if h.mma else []) + (["tma"] if h.tma else [])
    c = rng.choice(choices)
    if c == "mma":
      h.run_mma()
    elif c == "tma":
      h.land()
    elif not step(c) and not h.mma and not h.tma:
      # nothing in flight: unless some actor can move, this is a deadlock
      assert any(step(a) for a in list(actors)), "deadlock"
  else:
    raise AssertionError("no end in sight")
  assert h.s_read == [nkb] * 4


@pytest.mark.parametrize("nkb", [4, 5, 6, 7, 9, 16])
def test_attention_core_protocol_random_interleavings(nkb):
  for seed in range(60):
    simulate(nkb, seed, rescale_p=0.0 if seed % 3 == 0 else 0.3)


def test_model_catches_p_signalled_before_written():
  """The same model with one planted mistake (the softmax warps signal P_j before writing it)
  must fail: a model that passes everything proves nothing."""
  failures = 0
  for seed in range(30):
    try:
      simulate(7, seed, rescale_p=0.3, early_pready=True)
    except AssertionError:
      failures += 1
  assert failures > 10
