"""Host-side model of the multi-phase GEMM chain's synchronisation (csrc/gemm_w8a16.cu, w8a16_chain_kernel).

Each CTA's roles - TMA producer, dequant group, the NACC MMA issuers, the epilogue - are generators that wait on
mbarriers with hardware parity semantics (a wait for parity P succeeds once the barrier's current phase parity
differs from P, so a phase two generations old aliases like on the GPU), plus the grid barrier between phases.
Loads and MMA commits complete asynchronously in random order.  The rings, parities, issuer alternation and the
cross-phase weight prefetch follow the kernel; the model finding no deadlock for every pipeline shape and for odd
partitions (CTAs with 0/1/2 units per phase, more CTAs than units) is a check of the protocol, not of the hardware.
"""
import random

import pytest


class Bar:
    def __init__(s, name, count): s.name, s.count, s.arr, s.tx, s.phase = name, count, 0, 0, 0
    def done(s, parity): return (s.phase & 1) != parity
    def arrive(s):
        s.arr += 1; s._check()
    def expect(s, b): s.arr += 1; s.tx += b; s._check()
    def land(s, b): s.tx -= b; s._check()
    def _check(s):
        if s.arr >= s.count and s.tx == 0:
            s.phase += 1; s.arr -= s.count

def unit_start(c, U, G): return (c * U) // G

def sim(G, phases, RW, RX, F, NACC, fold, seed=0):
    rng = random.Random(seed)
    gbar = [0] * 5
    events = []   # pending async completions: (fn)
    roles = []
    for cta in range(G):
        wfull=[Bar('wfull',1) for _ in range(RW)]; wempty=[Bar('wempty',256) for _ in range(RW)]
        xfull=[Bar('xfull',1) for _ in range(RX)]; xempty=[Bar('xempty',1) for _ in range(RX)]
        ffull=[Bar('ffull',256) for _ in range(F)]; fempty=[Bar('fempty',1) for _ in range(F)]
        afull=[Bar('afull',NACC) for _ in range(2)]; aempty=[Bar('aempty',128) for _ in range(2)]
        def prod(cta=cta, wfull=wfull, wempty=wempty, xfull=xfull, xempty=xempty):
            sw=sx=0; pw=px=1
            for p,(tiles,kt) in enumerate(phases):
                U=tiles*kt; u0,u1=unit_start(cta,U,G),unit_start(cta+1,U,G); n=u1-u0
                pre = min(n,RW) if p>0 else 0
                def issue_w():
                    nonlocal sw,pw
                    b=wempty[sw]; par=pw
                    yield lambda: b.done(par)
                    wf=wfull[sw]; wf.expect(1); events.append(lambda wf=wf: wf.land(1))
                    sw+=1
                    if sw==RW: sw=0; pw^=1
                for i in range(pre):
                    yield from issue_w()
                if p>0:
                    yield lambda p=p: gbar[p-1] >= G
                for i in range(n):
                    if i>=pre: yield from issue_w()
                    b=xempty[sx]; par=px
                    yield lambda: b.done(par)
                    xf=xfull[sx]; xf.expect(1); events.append(lambda xf=xf: xf.land(1))
                    sx+=1
                    if sx==RX: sx=0; px^=1
        def mma(mw, cta=cta, xfull=xfull, xempty=xempty, ffull=ffull, fempty=fempty, afull=afull, aempty=aempty):
            seg=0; sx=f=0; phx=phf=0
            for p,(tiles,kt) in enumerate(phases):
                U=tiles*kt; u0,u1=unit_start(cta,U,G),unit_start(cta+1,U,G)
                u=u0
                while u<u1:
                    tile=u//kt; te=(tile+1)*kt; ue=min(te,u1); acc=seg&1
                    b=aempty[acc]; par=((seg>>1)&1)^1
                    yield lambda b=b,par=par: b.done(par)
                    for k in range(u,ue):
                        if (k-u0)%NACC != mw:
                            sx+=1
                            if sx==RX: sx=0; phx^=1
                            f+=1
                            if f==F: f=0; phf^=1
                            continue
                        if not fold:
                            b=xfull[sx]; par=phx
                            yield lambda b=b,par=par: b.done(par)
                        b=ffull[f]; par=phf
                        yield lambda b=b,par=par: b.done(par)
                        xe=xempty[sx]; fe=fempty[f]
                        events.append(lambda xe=xe: xe.arrive()); events.append(lambda fe=fe: fe.arrive())
                        sx+=1
                        if sx==RX: sx=0; phx^=1
                        f+=1
                        if f==F: f=0; phf^=1
                    af=afull[acc]; events.append(lambda af=af: af.arrive())
                    seg+=1; u=ue
        def dq(cta=cta, wfull=wfull, wempty=wempty, xfull=xfull, ffull=ffull, fempty=fempty):
            sw=f=sx=0; pw=0; pf=1; px=0
            for p,(tiles,kt) in enumerate(phases):
                U=tiles*kt; n=unit_start(cta+1,U,G)-unit_start(cta,U,G)
                for i in range(n):
                    b=wfull[sw]; par=pw
                    yield lambda b=b,par=par: b.done(par)
                    b=fempty[f]; par=pf
                    yield lambda b=b,par=par: b.done(par)
                    if fold:
                        b=xfull[sx]; par=px
                        yield lambda b=b,par=par: b.done(par)
                    for _ in range(256): wempty[sw].arrive()
                    for _ in range(256): ffull[f].arrive()
                    sw+=1
                    if sw==RW: sw=0; pw^=1
                    f+=1
                    if f==F: f=0; pf^=1
                    sx+=1
                    if sx==RX: sx=0; px^=1
        def epi(cta=cta, afull=afull, aempty=aempty):
            seg=0
            for p,(tiles,kt) in enumerate(phases):
                if p>0: yield lambda p=p: gbar[p-1] >= G
                U=tiles*kt; u0,u1=unit_start(cta,U,G),unit_start(cta+1,U,G)
                u=u0
                while u<u1:
                    tile=u//kt; te=(tile+1)*kt; ue=min(te,u1); acc=seg&1
                    b=afull[acc]; par=(seg>>1)&1
                    yield lambda b=b,par=par: b.done(par)
                    for _ in range(128): aempty[acc].arrive()
                    seg+=1; u=ue
                gbar[p]+=1
        roles += [(f"prod{cta}", prod()), (f"dq{cta}", dq()), (f"epi{cta}", epi())] + [(f"mma{cta}.{m}", mma(m)) for m in range(NACC)]
    # scheduler
    state = {name: (g, None) for name, g in roles}
    def step(name):
        g, pred = state[name]
        if pred is not None and not pred(): return False
        try:
            pred = next(g)
        except StopIteration:
            del state[name]; return True
        state[name] = (g, pred); return True
    names = list(state)
    while state:
        progressed = False
        for name in list(state):
            if name in state and step(name): progressed = True
        while events:
            rng.shuffle(events)
            e = events.pop(); e(); progressed = True
        if not progressed:
            stuck = sorted(state)[:12]
            return False, stuck
    return True, None



CFGS = {16: (4, 8, 3, 2, True), 32: (4, 4, 3, 2, True), 64: (4, 2, 2, 2, False), 128: (2, 2, 2, 1, False)}
SHAPES = [[(16, 16), (24, 8)], [(64, 32), (448, 32), (64, 112), (80, 32)], [(8, 2), (3, 5)], [(1, 1), (2, 3), (5, 1)]]


@pytest.mark.parametrize("bn", sorted(CFGS))
@pytest.mark.parametrize("shape", range(len(SHAPES)))
@pytest.mark.parametrize("G", [148, 7])
def test_chain_protocol_has_no_deadlock(bn, shape, G):
    RW, RX, F, NACC, fold = CFGS[bn]
    for seed in range(1 if G > 100 else 3):
        ok, stuck = sim(G, SHAPES[shape], RW, RX, F, NACC, fold, seed=seed)
        assert ok, stuck
