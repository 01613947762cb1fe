"""Model of the barrier protocol of the pair-transition kernel (k_transition_tc in
sparsefold_b200/csrc/sf_transition_tc.cu), run under many random interleavings on the CPU.

Actors of one CTA over several 256-position passes: the TMA producer (x tiles, W1 ring), the
two GEMM1 issuers (one per 128-position tile), the GEMM2 issuer (which also refills the W2
ring), the eight element-wise warps (four per tile: LayerNorm, then SwiGLU per chunk), the four
residual-epilogue warps (eight units per pass through two staging buffers, the first warp's
leader thread loading each unit's x rows and storing the sum), the tensor core (MMAs run one at
a time in issue order; a commit arrives once everything issued before it has run) and the TMA
engine (loads land in any order; a store reads its staging some time before its wait returns).
Every parity wait checks that its barrier is within one phase of the phase it waits for, and
every shared-memory stage, TMEM buffer and hidden buffer records what it holds, so a reader
that would see the wrong chunk, or a writer that would overwrite data still in use, fails.
"""
import random

import pytest

NCHUNK, W1S, W2S, HBUF = 16, 4, 4, 3


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
  def __init__(self, passes, rng, w2_early=False, early_reload=False):
    # w2_early plants a mistake in the model (a W2 stage refilled without waiting for the GEMM2
    # that reads it), early_reload another (a staging buffer reloaded before the store of its last
    # unit has read it), to show that the model catches them
    self.P, self.rng, self.w2_early, self.early_reload = passes, rng, w2_early, early_reload
    B = Bar
    self.xfull, self.xready, self.xfree = B("xfull", 2), B("xready", 8), B("xfree", 2)
    self.accfull, self.accfree = B("accfull", 1), B("accfree", 4)
    self.ybar = [B(f"ybar{i}", 2) for i in range(2)]
    self.ystage = [None, None]             # ("loading" | "x" | "sum" | "ydone", pass, unit)
    self.ysync = {}                        # (pass, unit) -> epilogue warps that wrote their rows
    self.w1full = [B(f"w1full{i}", 2) for i in range(W1S)]
    self.w1free = [B(f"w1free{i}", 2) for i in range(W1S)]
    self.w2full = [B(f"w2full{i}", 2) for i in range(W2S)]
    self.w2free = [B(f"w2free{i}", 1) for i in range(W2S)]
    self.s1full = [B(f"s1full{i}", 1) for i in range(4)]       # [buffer][tile]
    self.s1free = [B(f"s1free{i}", 4) for i in range(4)]
    self.hfull = [B(f"hfull{i}", 8) for i in range(HBUF)]
    self.hfree = [B(f"hfree{i}", 1) for i in range(HBUF)]
    self.x = None                          # ("raw" | "ln", pass) or ("loading", pass)
    self.w1 = [None] * W1S                 # chunk index held
    self.w2 = [None] * W2S
    self.s1 = [None] * 4                   # (buffer, tile) -> chunk q
    self.h = [None] * (2 * HBUF)           # (buffer, tile) -> chunk q
    self.acc_pass = None
    self.mma, self.tma = [], []
    self.ln_done = {}
    self.s1_read = {}

  # ---- producer: x tiles and the W1 ring ----
  def producer(self):
    q = 0
    for pi in range(self.P):
      if pi >= 1:
        while not self.xfree.ready(pi - 1):
          yield "xfree"
      self.xfull.arrive()
      self.x = ("loading", pi)
      self.tma.append(("x", pi, self.xfull))
      yield None
      for _ in range(NCHUNK):
        st = q % W1S
        if q >= W1S:
          while not self.w1free[st].ready(q // W1S - 1):
            yield "w1free"
        self.w1full[st].arrive()
        self.w1[st] = ("loading", q)
        self.tma.append(("w1", (st, q), self.w1full[st]))
        q += 1
        yield None

  # ---- GEMM1 issuer of tile t2 ----
  def gemm1(self, t2):
    q = 0
    for pi in range(self.P):
      while not self.xready.ready(pi):
        yield "xready"
      for hc in range(NCHUNK):
        st, sbuf = q % W1S, q & 1
        while not self.w1full[st].ready(q // W1S):
          yield "w1full"
        if q >= 2:
          while not self.s1free[sbuf * 2 + t2].ready((q >> 1) - 1):
            yield "s1free"
        self.mma.append(("g1", (t2, st, sbuf, q, pi)))
        self.mma.append(("commit", self.s1full[sbuf * 2 + t2]))
        self.mma.append(("commit", self.w1free[st]))
        if hc == NCHUNK - 1:
          self.mma.append(("commit", self.xfree))
        q += 1
        yield None

  # ---- GEMM2 issuer, which also refills the W2 ring ----
  def gemm2(self):
    total = self.P * NCHUNK

    def load_w2(c):
      st = c % W2S
      self.w2full[st].arrive()
      self.w2[st] = ("loading", c)
      self.tma.append(("w2", (st, c), self.w2full[st]))

    for c in range(min(W2S, total)):
      load_w2(c)
    yield None
    q = 0
    for pi in range(self.P):
      for hc in range(NCHUNK):
        st, hb = q % W2S, q % HBUF
        if q >= 1 and q - 1 + W2S < total:
          while not self.w2_early and not self.w2free[(q - 1) % W2S].ready((q - 1) // W2S):
            yield "w2free"
          load_w2(q - 1 + W2S)
          yield None
        if hc == 0 and pi >= 1:
          while not self.accfree.ready(pi - 1):
            yield "accfree"
        while not self.hfull[hb].ready(q // HBUF):
          yield "hfull"
        while not self.w2full[st].ready(q // W2S):
          yield "w2full"
        self.mma.append(("g2", (hb, st, q, pi, hc)))
        self.mma.append(("commit", self.hfree[hb]))
        self.mma.append(("commit", self.w2free[st]))
        q += 1
        yield None
      self.mma.append(("commit", self.accfull))
      yield None

  # ---- an element-wise warp (warps 4 t2 .. 4 t2 + 3 hold the rows of tile t2) ----
  def elementwise(self, w):
    t2 = w // 4
    q = 0
    for pi in range(self.P):
      while not self.xfull.ready(pi):
        yield "xfull"
      assert self.x == ("raw", pi), f"LN of pass {pi} sees {self.x}"
      self.ln_done[pi] = self.ln_done.get(pi, 0) + 1
      if self.ln_done[pi] == 8:
        self.x = ("ln", pi)
      self.xready.arrive()
      yield None
      for hc in range(NCHUNK):
        sbuf = q & 1
        while not self.s1full[sbuf * 2 + t2].ready(q >> 1):
          yield "s1full"
        assert self.s1[sbuf * 2 + t2] == q, f"element-wise warp reads S1 {self.s1[sbuf * 2 + t2]} for chunk {q}"
        self.s1free[sbuf * 2 + t2].arrive()
        yield None
        hbuf = q % HBUF
        if q >= HBUF:
          while not self.hfree[hbuf].ready(q // HBUF - 1):
            yield "hfree"
        cur = self.h[hbuf * 2 + t2]
        # free: never used, or a hidden tile GEMM2 is done with (or this chunk, written by another
        # warp of the tile: each warp writes its own rows)
        assert cur is None or cur[1] <= q - HBUF or cur[1] == q, f"chunk {q} hidden write over {cur}"
        self.h[hbuf * 2 + t2] = ("h", q)
        self.hfull[hbuf].arrive()
        q += 1
        yield None

  # ---- a residual-epilogue warp; warp 0's leader also loads and stores the units ----
  def load_unit(self, pi, u):
    b = u & 1
    assert self.ystage[b] is None or self.ystage[b][0] == "ydone", f"unit ({pi}, {u}) loaded over {self.ystage[b]}"
    self.ybar[b].arrive()
    self.ystage[b] = ("loading", pi, u)
    self.tma.append(("yload", (b, pi, u), self.ybar[b]))

  def epilogue(self, e):
    for pi in range(self.P):
      if e == 0:
        self.load_unit(pi, 0)
        self.load_unit(pi, 1)
        yield None
      while not self.accfull.ready(pi):
        yield "accfull"
      for u in range(8):
        assert self.acc_pass == pi, f"epilogue of pass {pi} reads the accumulators of {self.acc_pass}"
        if u == 7:
          self.accfree.arrive()
        b = u & 1
        while not self.ybar[b].ready(pi * 4 + (u >> 1)):
          yield "ybar"
        assert self.ystage[b] in (("x", pi, u), ("sum", pi, u)), f"unit ({pi}, {u}) reads staging {self.ystage[b]}"
        self.ysync.setdefault((pi, u), set()).add(e)
        yield None
        while len(self.ysync[(pi, u)]) < 4:     # the epilogue warps' named barrier
          yield "ysync"
        if e == 0:
          self.ystage[b] = ("sum", pi, u)
          self.tma.append(("ystore", (b, pi, u), None))
          yield None
          if not self.early_reload:
            while self.ystage[b] != ("ydone", pi, u):   # bulk wait: the store has read the staging
              yield "ystore"
          if u + 2 < 8:
            self.load_unit(pi, u + 2)
          yield None

class Sim:
  def __init__(self, passes, seed, w2_early=False, early_reload=False):
    self.rng = random.Random(seed)
    self.c = Cta(passes, self.rng, w2_early, early_reload)

  def run_mma(self):
    c = self.c
    kind, arg = c.mma.pop(0)
    if kind == "g1":
      t2, st, sbuf, q, pi = arg
      assert c.x == ("ln", pi), f"GEMM1 chunk {q} reads x {c.x}"
      assert c.w1[st] == q, f"GEMM1 chunk {q} reads W1 stage {c.w1[st]}"
      prev = c.s1[sbuf * 2 + t2]
      assert prev is None or prev == q - 2, f"GEMM1 chunk {q} overwrites S1 of chunk {prev}"
      c.s1[sbuf * 2 + t2] = q
    elif kind == "g2":
      hb, st, q, pi, hc = arg
      assert c.h[hb * 2] == ("h", q) and c.h[hb * 2 + 1] == ("h", q), f"GEMM2 chunk {q} reads {c.h[hb * 2:hb * 2 + 2]}"
      assert c.w2[st] == q, f"GEMM2 chunk {q} reads W2 stage {c.w2[st]}"
      if hc == 0:
        c.acc_pass = pi
    else:
      arg.arrive()

  def land(self):
    c = self.c
    kind, arg, bar = c.tma.pop(self.rng.randrange(len(c.tma)))
    if kind == "yload":
      b, pi, u = arg
      assert c.ystage[b] == ("loading", pi, u), f"unit ({pi}, {u}) lands over {c.ystage[b]}"
      c.ystage[b] = ("x", pi, u)
    elif kind == "ystore":
      b, pi, u = arg
      assert c.ystage[b] == ("sum", pi, u), f"the store of unit ({pi}, {u}) reads {c.ystage[b]}"
      c.ystage[b] = ("ydone", pi, u)
      return
    elif kind == "x":
      c.x = ("raw", arg)
    elif kind == "w1":
      st, q = arg
      c.w1[st] = q
    else:
      st, q = arg
      c.w2[st] = q
    bar.arrive()


def simulate(passes, seed, w2_early=False, early_reload=False):
  s = Sim(passes, seed, w2_early, early_reload)
  c = s.c
  gens = ([c.producer(), c.gemm1(0), c.gemm1(1), c.gemm2()] + [c.elementwise(w) for w in range(8)] +
          [c.epilogue(e) for e in range(4)])
  actors = dict(enumerate(gens))

  def step(a):
    try:
      return next(actors[a]) is None
    except StopIteration:
      del actors[a]
      return True

  for _ in range(2000000):
    if not actors and not c.mma and not c.tma:
      break
    choices = list(actors) + (["mma"] if c.mma else []) + (["tma"] if c.tma else [])
    ch = s.rng.choice(choices)
    if ch == "mma":
      s.run_mma()
    elif ch == "tma":
      s.land()
    elif not step(ch) and not c.mma and not c.tma:
      assert any(step(a) for a in list(actors)), "deadlock"
  else:
    raise AssertionError("no end in sight")


@pytest.mark.parametrize("passes", [1, 2, 3])
def test_transition_protocol_random_interleavings(passes):
  for seed in range(12):
    simulate(passes, seed)


def test_model_catches_early_w2_refill():
  """The same model with one planted mistake must fail."""
  failures = 0
  for seed in range(10):
    try:
      simulate(2, seed, w2_early=True)
    except AssertionError:
      failures += 1
  assert failures >= 8


def test_model_catches_a_staging_reload_before_its_store_has_read_it():
  """The residual epilogue with its bulk wait removed must fail."""
  failures = 0
  for seed in range(20):
    try:
      simulate(2, seed, early_reload=True)
    except AssertionError:
      failures += 1
  assert failures >= 5, failures
