"""Model of the barrier protocol of the generic attention kernel (k_mha_tc in
sparsefold_b200/csrc/sf_attn_tc.cu), run under many random interleavings on the CPU.

Actors: the TMA producer thread (a 3-slot ring of K/V/bias tiles; the first slots are requested
before the CTA-wide barrier, later ones after the slot's P V is done), the MMA issuer thread, the
four softmax warps, the tensor core (MMAs run one at a time in issue order; a commit arrives once
everything issued before it has run) and the TMA engine (loads land in any order).  As in the model
of the triangle-attention core, every parity wait checks that its barrier has completed exactly the
phases before the one waited for or one more, ring slots and TMEM buffers carry the block they hold,
and each reader checks it sees the block it expects.  The kernel's one irregular barrier is
``pready[1]``: its first phase says "Q is in TMEM", so key block j waits on phase (j >> 1) + (j & 1)
of ``pready[j & 1]``.
"""
import random

import pytest

RING = 3


class Bar:
  def __init__(self, name, count):
    self.name, self.count, self.arrived, self.done = name, count, 0, 0

  def arrive(self):
    self.arrived += 1
    assert self.arrived <= self.count, f"{self.name}: too many arrivals"
    if self.arrived == self.count:
      self.arrived, self.done = 0, self.done + 1

  def ready(self, use):
    assert self.done in (use, use + 1), f"{self.name}: waiting for use {use} with {self.done} phases complete"
    return self.done == use + 1


class Cta:
  def __init__(self, nkb, rng, rescale_p, planted=None):
    self.nkb, self.rng, self.rescale_p, self.planted = nkb, rng, rescale_p, planted
    self.kvfull = [Bar(f"kvfull{i}", 2) for i in range(RING)]   # expect_tx arrival + the bytes landing
    self.kvfree = [Bar(f"kvfree{i}", 1) for i in range(RING)]
    self.sbar = [Bar(f"sbar{i}", 2) for i in range(2)]          # issuer's arrival + the S commit
    self.pready = [Bar(f"pready{i}", 4) for i in range(2)]
    self.pvbar = [Bar(f"pvbar{i}", 1) for i in range(2)]
    self.slot = [None] * RING      # block whose K, V and bias tiles the slot holds
    self.tmem = [None, None]       # S/P buffers: ("S", j) or ("P", j)
    self.q_in_tmem = False
    self.mma, self.tma = [], []
    self.pv_done = set()
    self.s_read = [0] * 4
    self.p_written = {}

  # ---- TMA producer ----
  def load(self, jj):
    bar = self.kvfull[jj % RING]
    bar.arrive()   # expect_tx
    self.slot[jj % RING] = ("loading", jj)
    self.tma.append((jj % RING, jj, bar))

  def producer(self):
    for jj in range(min(RING, self.nkb)):   # before the CTA barrier
      self.load(jj)
    yield None
    for jj in range(RING, self.nkb):
      if self.planted != "refill_early":
        while not self.kvfree[jj % RING].ready(jj // RING - 1):
          yield ("kvfree", jj)
      self.load(jj)
      yield None

  # ---- MMA issuer ----
  def issuer(self):
    nkb = self.nkb

    def issue_s(jj):
      while not self.kvfull[jj % RING].ready(jj // RING):
        yield ("kvfull", jj)
      self.sbar[jj & 1].arrive()
      self.mma.append(("S", jj))
      self.mma.append(("commit", self.sbar[jj & 1]))
      yield None

    while not self.pready[1].ready(0):   # Q is in TMEM
      yield ("q", None)
    yield from issue_s(0)
    if nkb > 1:
      yield from issue_s(1)
    for j in range(nkb):
      ph = (j >> 1) if self.planted == "no_q_phase" else (j >> 1) + (j & 1)
      while not self.pready[j & 1].ready(ph):
        yield ("pready", j)
      self.mma.append(("PV", j))
      self.mma.append(("commit", self.pvbar[j & 1]))
      self.mma.append(("commit", self.kvfree[j % RING]))
      yield None
      if j + 2 < nkb:
        yield from issue_s(j + 2)

  # ---- a softmax warp ----
  def softmax(self, w):
    nkb = self.nkb
    self.q_in_tmem = True
    self.pready[1].arrive()   # Q in TMEM
    yield None
    for j in range(nkb):
      while not self.sbar[j & 1].ready(j >> 1):
        yield ("sbar", j)
      assert self.tmem[j & 1] == ("S", j), f"softmax {w} block {j} reads {self.tmem[j & 1]}"
      assert self.slot[j % RING] == j, f"softmax {w} block {j} bias tile holds {self.slot[j % RING]}"
      self.s_read[w] += 1
      yield None
      if j >= 1 and self.rng.random() < self.rescale_p:   # the running max moved: rescale O
        while not self.pvbar[(j - 1) & 1].ready((j - 1) >> 1):
          yield ("pvbar", j - 1)
        assert (j - 1) in self.pv_done
      assert self.tmem[j & 1] in (("S", j), ("P", j)), f"softmax {w} writes P_{j} over {self.tmem[j & 1]}"
      self.p_written.setdefault(j, set()).add(w)
      if len(self.p_written[j]) == 4:
        self.tmem[j & 1] = ("P", j)
      self.pready[j & 1].arrive()
      yield None
    for jj in (nkb - 2, nkb - 1):
      if jj >= 0:
        while not self.pvbar[jj & 1].ready(jj >> 1):
          yield ("pvbar-end", jj)
    assert all(j in self.pv_done for j in range(nkb))

  # ---- tensor core and TMA engine ----
  def run_mma(self):
    kind, arg = self.mma.pop(0)
    if kind == "S":
      assert self.q_in_tmem
      assert self.slot[arg % RING] == arg, f"S_{arg} reads K slot {self.slot[arg % RING]}"
      prev = self.tmem[arg & 1]
      assert prev is None or (prev == ("P", arg - 2) and (arg - 2) in self.pv_done), f"S_{arg} overwrites {prev}"
      self.tmem[arg & 1] = ("S", arg)
    elif kind == "PV":
      assert self.tmem[arg & 1] == ("P", arg), f"PV_{arg} reads {self.tmem[arg & 1]}"
      assert self.slot[arg % RING] == arg, f"PV_{arg} reads V slot {self.slot[arg % RING]}"
      self.pv_done.add(arg)
    else:
      arg.arrive()

  def land(self):
    idx, val, bar = self.tma.pop(self.rng.randrange(len(self.tma)))
    self.slot[idx] = val
    bar.arrive()


def simulate(nkb, seed, rescale_p, planted=None):
  rng = random.Random(seed)
  c = Cta(nkb, rng, rescale_p, planted)
  gens = [c.producer(), c.issuer()] + [c.softmax(w) for w in range(4)]
  actors = dict(enumerate(gens))

  def step(a):
    try:
      return next(actors[a]) is None
    except StopIteration:
      del actors[a]
      return True

  for _ in range(400000):
    if not actors and not c.mma and not c.tma:
      break
    choices = list(actors) + (["mma"] if c.mma else []) + (["tma"] if c.tma else [])
    ch = rng.choice(choices)
    if ch == "mma":
      c.run_mma()
    elif ch == "tma":
      c.land()
    elif not step(ch) and not c.mma and not c.tma:
      assert any(step(a) for a in list(actors)), "deadlock"
  else:
    raise AssertionError("no end in sight")
  assert c.s_read == [nkb] * 4


@pytest.mark.parametrize("nkb", [1, 2, 3, 4, 5, 8, 13])
def test_attention_kernel_protocol_random_interleavings(nkb):
  for seed in range(60):
    simulate(nkb, seed, rescale_p=0.0 if seed % 3 == 0 else 0.3)


@pytest.mark.parametrize("planted", ["no_q_phase", "refill_early"])
def test_model_catches_planted_mistakes(planted):
  """Two planted mistakes must fail: waiting on pready without the extra "Q in TMEM" phase (P V issued
  before P is written), and refilling a ring slot without waiting for its P V."""
  failures = 0
  for seed in range(30):
    try:
      simulate(7, seed, rescale_p=0.3, planted=planted)
    except AssertionError:
      failures += 1
  assert failures > 10
