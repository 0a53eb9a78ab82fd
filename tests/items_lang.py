"""Item functions written against tallymap_b200.lang, the traced counterparts of the hand-lowered items (the
reference's examples/quickstart.py:19-30 walker and benchmark configuration 2's walk), plus an item that exercises the other
lowered primitives.  Shared by the lowering tests."""
from tallymap_b200 import lang as tl


def quickstart(t, x, key, theta):
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        t = t.add("hist", (x * 16).astype(tl.int32), theta * (1 - x))
        return k + 1, x * (0.5 + 0.5 * u), t
    k, x, t = tl.while_loop(lambda c: c[1] > 0.05, body, (0, x, t))
    return t, k


def walk(t, x, key, drift):
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        t = t.add("hist", (x * 256).astype(tl.int32), drift * x)
        return k + 1, x + 0.02 * (2 * u - 1), t
    k, x, t = tl.while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1), body, (0, x, t))
    t = t.add("side", (x > 1).astype(tl.int32), 1.0)
    return t, k


def mixer(t, pos, key, n, a, b):
    """a fixed number of steps n (per item) so the outputs are smooth in the broadcast a and b: transcendentals,
    select, min/max, a 3-D tuple-indexed tally, an int tally, a per-item vector"""
    x0, y0, z0 = pos
    def body(c):
        k, x, y, w, t = c
        kk = tl.random.fold_in(key, k)
        u, v = tl.random.uniform(kk, (2,))
        s = -tl.log(1.0 - u) / (a + b)
        ang = 6.2831853 * v
        x = x + s * tl.cos(ang) * tl.sqrt(w)
        y = y + s * tl.sin(ang)
        w = tl.where(u < 0.5, w * tl.exp(-a * s), tl.minimum(w * 1.5, tl.maximum(w, 0.25)))
        ix = (x + 4.0).astype(tl.int32)
        iy = (y + 4.0).astype(tl.int32)
        iz = (k // 2) % 8
        t = t.add("dep", (ix, iy, iz), w * tl.power(b, 0.5) + a * x * y)
        t = t.add("hits", (k % 4,), 1)
        return k + 1, x, y, w, t
    k, x, y, w, t = tl.while_loop(lambda c: c[0] < n, body, (0, x0, y0 + z0, 1.0, t))
    t = t.add("end", 0, x * a - y * b + w)
    return t, k


def walk_records(t, x, key, drift):
    """the walk, recording each step that starts in bin 128 (step, position) and each item's exit (steps, side)"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        b = (x * 256).astype(tl.int32)
        t = t.add("hist", b, drift * x)
        t = t.append("hits", {"k": k, "x": x}, when=b == 128)
        return k + 1, x + 0.02 * (2 * u - 1), t
    k, x, t = tl.while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1), body, (0, x, t))
    t = t.append("exit", {"k": k, "side": (x > 1).astype(tl.int32)})
    return t, k


def edges(t, a, key, n, s):
    """every lowered primitive on awkward values (NaN, +-inf, -0, huge, negative integers), its results recorded so
    that they compare bitwise: a fixed number n of steps per item"""
    def body(c):
        k, x, t = c
        kk = tl.random.fold_in(key, k)
        u = tl.random.uniform(kk)
        b = tl.random.bits(kk, (2,))
        xi = x.astype(tl.int32)
        q = (xi - 7) // 3
        r = (xi - 7) % 3
        y = tl.where(x > 0.5, tl.log(x), tl.exp(-x * s)) + tl.power(u + 0.5, s)
        z = tl.minimum(tl.maximum(tl.sin(x * u), -0.0), tl.abs(tl.cos(y))) - tl.floor(x * 0.3) + tl.sqrt(u)
        t = t.append("rec", {"i": xi, "q": q, "r": r, "b": (b[0] ^ (b[1] >> 3)).astype(tl.int32), "y": y, "z": z,
                             "u": (x * 1e30).astype(tl.uint32).astype(tl.int32)})
        t = t.add("h", (q % 8,), 1)
        return k + 1, x * (1.5 - u) - 3.0 * s, t
    k, x, t = tl.while_loop(lambda c: c[0] < n, body, (0, a, t))
    return t, k


def shower(t, E, depth, key, X0):
    """benchmark configuration 5's branching shower as a tallymap user writes it: one particle per item; a split particle
    ends, replaced by two children spawned with the same per-item structure (energy, depth, key)"""
    def body(c):
        k, E, depth, alive, t = c
        kk = tl.random.fold_in(key, k)
        u = tl.random.uniform(kk, (3,))
        depth = depth + X0 * -tl.log(1.0 - u[0])
        low = E < 0.5
        t = t.add("dep", tl.where(low, (depth * 8).astype(tl.int32), 0), tl.where(low, E, 0.0))
        split = ~low & (u[1] < 0.7)
        z = 0.1 + 0.8 * u[2]
        t = t.spawn((E * z, depth, tl.random.fold_in(kk, 0)), when=split)
        t = t.spawn((E * (1.0 - z), depth, tl.random.fold_in(kk, 1)), when=split)
        return k + 1, E, depth, ~low & ~split, t
    k, E, depth, alive, t = tl.while_loop(lambda c: c[3], body, (0, E, depth, True, t))
    t = t.add("count", 0, 1)
    return t, k


def spawn_walk(t, g, x, key):
    """a divergent walk that spawns one child (generation g + 1) AFTER its loop while g < 3 (the reference's
    tests/invariants.py spawn_walk, with a random step): the post-loop spawn point"""
    def body(c):
        k, w, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        return k + 1, w * (0.5 + 0.5 * u), t.add("Q", k % 16, w).add("C", k % 16, 1)
    n = 2 + g + (x > 1.0).astype(tl.int32)
    k, w, t = tl.while_loop(lambda c: c[0] < n, body, (0, x, t))
    t = t.spawn((g + 1, w * 1.25, tl.random.fold_in(key, 7)), when=g < 3)
    return t, k


def spawn_decay(t, g, w, key, a):
    """three steps per item, each depositing a * w * u; a child (generation g + 1) with weight w * a after the loop
    while g < 2: the outputs are polynomials in the broadcast a (degree <= 3), so a central difference is exact up to
    its third-order term"""
    def body(c):
        k, w, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        t = t.add("Q", k % 8, a * w * u)
        return k + 1, w * 0.9, t
    k, w, t = tl.while_loop(lambda c: c[0] < 3, body, (0, w, t))
    t = t.spawn((g + 1, w * a, tl.random.fold_in(key, 7)), when=g < 2)
    return t, k


def scatter(t, x, key, a):
    """a loop-free item (no while_loop: the reference's 'item' schedule; here a loop of zero steps): two draws, two
    emits, a per-item result"""
    u, v = tl.random.uniform(key, (2,))
    t = t.add("h", ((x + u) * 4).astype(tl.int32), a * x * v)
    t = t.add("s", 0, tl.exp(-a * u))
    return t, x * 2 + u


def extras(t, a, key, n, s):
    """the compositions of lowered primitives (clip, sign, square, bernoulli) on awkward values, recorded so that they
    compare bitwise"""
    def body(c):
        k, x, t = c
        kk = tl.random.fold_in(key, k)
        u = tl.random.uniform(kk)
        hit = tl.random.bernoulli(kk, 0.3)
        y = tl.clip(x * s, -2.0, 3.0)
        z = tl.sign(x) * tl.square(u - 0.5) + tl.sign(tl.floor(x * 0.5)).astype(tl.float32)
        t = t.append("rec", {"y": y, "z": z, "h": hit.astype(tl.int32), "g": tl.sign((x * 3.0).astype(tl.int32))})
        return k + 1, x * (1.5 - u) - 0.25, t
    k, x, t = tl.while_loop(lambda c: c[0] < n, body, (0, a, t))
    return t, k


def affine(t, x, key, a):
    """n = 6 steps of x <- x * a + u, emitting x^2 at bin k % 8: smooth in the per-item x and the broadcast a, so its
    per-item gradient has a closed form (d x_k / d x_0 = a^k)"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        x = x * a + u
        t = t.add("h", k % 8, x * x)
        return k + 1, x, t
    k, x, t = tl.while_loop(lambda c: c[0] < 6, body, (0, x, t))
    return t, x


def rounding(t, a, key, n, s):
    """round, rem, mod and the vector reductions on awkward values, recorded so that they compare bitwise"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        v = (x * s, u - 0.5, x * u)
        t = t.append("rec", {"r": tl.round(x * 2.5), "m": tl.rem(x, s + u), "o": tl.mod(x, u - 0.6),
                             "s": tl.sum(v), "x": tl.max(v), "n": tl.min(v),
                             "a": (tl.all((x > 0.0, u > 0.5)) | tl.any((x < -5.0, u < 0.1))).astype(tl.int32)})
        return k + 1, x * (1.5 - u) - 0.75, t
    k, x, t = tl.while_loop(lambda c: c[0] < n, body, (0, a, t))
    return t, k


def stopped(t, x, key, a):
    """rem and stop_gradient in the emitted value: d/da = x (rem's derivative in its first argument is 1, the
    stopped term contributes nothing)"""
    t = t.add("h", 0, tl.rem(x * a, 0.7) + tl.stop_gradient(a) * x)
    return t, x


def transcend(t, x, key, s):
    """log1p, expm1 and tanh (compositions: Goldberg's and Kahan's methods), recorded"""
    t = t.append("rec", {"l": tl.log1p(x), "e": tl.expm1(x * s), "h": tl.tanh(x)})
    return t, x


def birth_death(t, x0, key, c0, c1):
    """an exact stochastic simulation (Gillespie's direct method) of a birth-death process: X -> X + 1 at rate
    c[0] * 50, X -> X - 1 at rate c[1] * X; run to time 2, the final count tallied into a histogram, the mean time
    step and the event count per item"""
    def body(s):
        k, tt, x, t = s
        xf = x.astype(tl.float32)
        a = (tl.maximum(c0 * 50.0, 0.0), tl.maximum(c1 * xf, 0.0))
        a0 = tl.sum(a)
        u = tl.random.uniform(tl.random.fold_in(key, k), (2,))
        tau = -tl.log(tl.maximum(u[0], 1e-20)) / tl.maximum(a0, 1e-20)
        r = tl.clip(tl.searchsorted(tl.cumsum(a), u[1] * a0, side="right"), 0, 1)
        x = tl.clip(x + tl.where(r == 0, 1, -1), 0, 1000)
        t = t.add("tau", 0, tau)
        return k + 1, tt + tau, x, t
    k, tt, x, t = tl.while_loop(lambda s: s[1] < 2.0, body, (0, 0.0, x0, t))
    t = t.add("hist", tl.clip(x // 8, 0, 31), 1)
    return t, x, k


def divided(t, x, key, a):
    """a walk whose control flow has no division or square root; the values it tallies divide and take roots"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        t = t.add("h", tl.clip((x * 16).astype(tl.int32), 0, 15), tl.sqrt(u) / (a + x))
        return k + 1, x + 0.05 * (2 * u - 1), t
    k, x, t = tl.while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1), body, (0, x, t))
    return t, k


def walk_theta(t, x, key, theta):
    """the 1-D walk with its parameters as one broadcast vector: theta = (drift weight, step, bias)"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        t = t.add("hist", tl.clip((x * 64).astype(tl.int32), 0, 63), theta[0] * x + theta[2])
        return k + 1, x + theta[1] * (2 * u - 1), t
    k, x, t = tl.while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1), body, (0, x, t))
    return t, k


def walk_theta_scalars(t, x, key, w, step, bias):
    """walk_theta with its three parameters as separate broadcast scalars"""
    return walk_theta(t, x, key, (w, step, bias))


def lookup(t, x, key, xs, pairs, a):
    """a walk reading its step size from a 1-D table and a pair of values from a 2-D (n, 2) table, by traced
    indices that leave the tables' range (clamped) and go negative (counted from the end, then clamped)"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        b = (x * 100).astype(tl.int32)
        sig = xs[b]
        lo, hi = pairs[b - 3]
        t = t.add("h", tl.clip(b // 8, 0, 15), a * sig * (hi - lo))
        return k + 1, x + 0.05 * (2 * u - 1) * sig, t
    k, x, t = tl.while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1), body, (0, x, t))
    return t, k, xs[-1] + pairs[k, 1]


def neighbours(t, i, order, start, pos, theta):
    """ONE particle of a cell list (a square box of side 8 in 4 x 4 cells, periodic): visit the members of the 3 x 3
    cells around particle i, one per loop step, summing a pair energy theta[0] * exp(-r^2 / theta[1]) over those
    within distance 2; tally half of it by the particle's column and return its neighbour count and energy"""
    xi, yi = pos[i]
    cx = tl.clip((xi / 2.0).astype(tl.int32), 0, 3)
    cy = tl.clip((yi / 2.0).astype(tl.int32), 0, 3)

    def body(c):
        g, p, nb, u, t = c
        cid = ((cy + g // 3 + 3) % 4) * 4 + (cx + g % 3 + 3) % 4
        lo, hi = start[cid], start[cid + 1]
        p = tl.maximum(p, lo)
        inside = p < hi
        j = order[p]
        xj, yj = pos[j]
        dx = tl.rem(xj - xi + 12.0, 8.0) - 4.0
        dy = tl.rem(yj - yi + 12.0, 8.0) - 4.0
        r2 = dx * dx + dy * dy
        near = inside & (j != i) & (r2 < 4.0)
        e = tl.where(near, theta[0] * tl.exp(-r2 / theta[1]), 0.0)
        nxt = p + 1
        done = ~(nxt < hi)
        return g + done.astype(tl.int32), tl.where(done, 0, nxt), nb + near.astype(tl.int32), u + e, t
    g, p, nb, u, t = tl.while_loop(lambda c: c[0] < 9, body, (0, 0, 0, 0.0, t))
    t = t.add("u", cx, 0.5 * u)
    return t, nb, u


def special(t, x, key, a):
    """every math primitive beyond log / exp / sin / cos, on values inside their domains, with the normal and
    exponential samplers: the per-item sum is tallied, and returned with a few of the values"""
    def body(c):
        k, s, t = c
        kk = tl.random.fold_in(key, k)
        z = tl.random.normal(kk)
        e = tl.random.exponential(tl.random.fold_in(kk, 7))
        u = tl.random.uniform(tl.random.fold_in(kk, 9), minval=-0.9, maxval=0.9)
        v = (tl.arctan(a * x + z) + tl.arctan2(z, a + u) + tl.arcsin(u * a * 0.5) + tl.arccos(u) + tl.tan(u)
             + tl.sinh(u * a) + tl.cosh(u) + tl.arcsinh(z * a) + tl.arccosh(1.5 + e * a) + tl.arctanh(u)
             + tl.exp2(u * a) + tl.log2(1.0 + e) + tl.cbrt(z * a) + tl.erf(z * a) + tl.erfc(u + a)
             + tl.erfinv(u * 0.9) + tl.log10(1.0 + e) + tl.logistic(z) + tl.ceil(u * 4.0))
        t = t.add("h", (tl.clip(u * 4.0 + 4.0, 0.0, 7.0)).astype(tl.int32), v * 0.01)
        return k + 1, s + v, t
    k, s, t = tl.while_loop(lambda c: c[0] < 6, body, (0, x, t))
    return t, s, tl.isfinite(s).astype(tl.int32)


def branchy(t, x, key, a):
    """a walk whose step is chosen by lax.cond and lax.switch and smoothed by a static fori_loop"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        dx = tl.cond(u < 0.5, lambda v: -a * v, lambda v: a * (1.0 - v), u)
        w = tl.switch((u * 3.0).astype(tl.int32), [lambda v: v, lambda v: v * v, lambda v: tl.sqrt(v)], u)
        w = tl.fori_loop(0, 2, lambda i, s: s * 0.5 + w, w)
        t = t.add("h", tl.clip((x * 8).astype(tl.int32), 0, 7), w * a)
        return k + 1, x + 0.1 * dx, t
    k, x, t = tl.while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1), body, (0, x, t))
    return t, k


def spheres(t, x0, point, key, theta):
    """a walk-on-spheres estimator for the Poisson problem on the unit square written with jax.numpy-style vectors
    (the reference's examples/walk_on_spheres.py problem): a source theta0 exp(-theta1 |y - 1/2|^2) sampled in each
    ball, boundary values theta2 + theta3 cos(2 pi (x + y)); the estimate tallied at the walker's point"""
    def dist(x):
        return tl.minimum(tl.minimum(x[0], 1.0 - x[0]), tl.minimum(x[1], 1.0 - x[1]))

    def body(c):
        x, acc, k = c
        R = dist(x)
        u = tl.random.uniform(tl.random.fold_in(key, k), (3,))
        r, a = R * tl.sqrt(u[0]), 2.0 * tl.pi * u[1]
        y = x + r * tl.array([tl.cos(a), tl.sin(a)])
        src = theta[0] * tl.exp(-theta[1] * tl.sum((y - 0.5) ** 2))
        acc = acc - 0.25 * R * R * tl.log(tl.maximum(u[0], 1e-20)) * src
        a2 = 2.0 * tl.pi * u[2]
        return x + R * tl.stack([tl.cos(a2), tl.sin(a2)]), acc, k + 1
    x, acc, k = tl.while_loop(lambda c: dist(c[0]) > 1e-3, body, (x0, 0.0, 0))
    est = acc + theta[2] + theta[3] * tl.cos(2.0 * tl.pi * (x[0] + x[1]))
    return t.add("u", point, est), k


def drift2d(t, x0, key, a):
    """a 2-D walk in the unit square returning its exit point as a vector and its step count"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k), (2,))
        return k + 1, x + a * (2.0 * u - 1.0), t
    inside = lambda x: (x[0] > 0.0) & (x[0] < 1.0) & (x[1] > 0.0) & (x[1] < 1.0)
    k, x, t = tl.while_loop(lambda c: inside(c[1]), body, (0, x0, t))
    t = t.add("exits", (x[0] > 1.0).astype(tl.int32) + 2 * (x[1] > 1.0).astype(tl.int32), 1.0)
    return t, x, k


def decay_records(t, w, key, a):
    """six steps per item; a step records (step, a * weight) when its draw is below 0.6, and the item's final
    (weight, steps): every recorded value is a polynomial in the broadcast a, the number of records is not a
    function of a (Records outputs under forward and reverse mode)"""
    def body(c):
        k, w, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        t = t.append("hits", {"k": k, "w": w * a}, when=u < 0.6)
        t = t.add("tot", 0, w)
        return k + 1, w * (0.5 + 0.4 * u) * a, t
    k, w, t = tl.while_loop(lambda c: c[0] < 6, body, (0, w, t))
    t = t.append("last", {"k": k, "w": w})
    return t, k


def pre_records(t, w, key, a):
    """records before the loop, in it and after it into one output (the item's ordinals in that order)"""
    t = t.append("log", {"k": -1, "w": w * a})
    def body(c):
        k, w, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        t = t.append("log", {"k": k, "w": w}, when=u < 0.5)
        return k + 1, w * (0.6 + 0.3 * u) * a, t
    k, w, t = tl.while_loop(lambda c: c[0] < 4, body, (0, w, t))
    t = t.append("log", {"k": 99, "w": w * w})
    return t, k


# Dormand-Prince 5(4): the tableau as Python floats (each rounded once to f32 where it meets an f32 value)
_DP_A = ((1 / 5,), (3 / 40, 9 / 40), (44 / 45, -56 / 15, 32 / 9),
         (19372 / 6561, -25360 / 2187, 64448 / 6561, -212 / 729),
         (9017 / 3168, -355 / 33, 46732 / 5247, 49 / 176, -5103 / 18656))
_DP_B = (35 / 384, 500 / 1113, 125 / 192, -2187 / 6784, 11 / 84)          # of k1, k3, k4, k5, k6
_DP_E = (71 / 57600, -71 / 16695, 71 / 1920, -17253 / 339200, 22 / 525, -1 / 40)   # of k1, k3 .. k7


def lorenz(t, sigma, rho, y0, item_id, beta):
    """benchmark configuration 4's item as a tallymap user writes it (the hand-lowered csrc/items_ode.cuh states the
    same source): Lorenz systems integrated by adaptive Dormand-Prince 5(4) on t in [0, 10], every linear
    combination summed left to right"""
    def f(y):
        return (sigma * (y[1] - y[0]), y[0] * (rho - y[2]) - y[1], y[0] * y[1] - beta * y[2])

    def lin(cs, ks, j):
        acc = cs[0] * ks[0][j]
        for c, k in zip(cs[1:], ks[1:]):
            acc = acc + c * k[j]
        return acc

    def axpy(y, hh, d):
        return tuple(y[j] + hh * d[j] for j in range(3))

    def body(c):
        k, tt, h, ya, yb, yc, ka, kb, kc, t = c
        y, k1 = (ya, yb, yc), (ka, kb, kc)
        hh = tl.minimum(h, 10.0 - tt)
        ks = [k1]
        for row in _DP_A:
            ks.append(f(axpy(y, hh, tuple(lin(row, ks, j) for j in range(3)))))
        k1_, k2, k3, k4, k5, k6 = ks
        y5 = axpy(y, hh, tuple(lin(_DP_B, (k1_, k3, k4, k5, k6), j) for j in range(3)))
        k7 = f(y5)
        e = tuple(hh * lin(_DP_E, (k1_, k3, k4, k5, k6, k7), j) for j in range(3))
        q = tuple(e[j] / (1e-9 + 1e-6 * tl.maximum(tl.abs(y[j]), tl.abs(y5[j]))) for j in range(3))
        err = tl.sqrt((q[0] * q[0] + q[1] * q[1] + q[2] * q[2]) / 3.0)
        ok = err <= 1.0
        fac = tl.stop_gradient(tl.clip(0.9 * err ** -0.2, 0.2, 10.0))
        yn = tuple(tl.where(ok, y5[j], y[j]) for j in range(3))
        kn = tuple(tl.where(ok, k7[j], k1[j]) for j in range(3))
        return (k + 1, tl.where(ok, tt + hh, tt), hh * fac) + yn + kn + (t,)
    y = (y0[0], y0[1], y0[2])
    c = tl.while_loop(lambda c: c[1] < 10.0, body, (0, 0.0, 1e-3) + y + f(y) + (t,))
    k, yf, t = c[0], c[3:6], c[9]
    for j in range(3):
        t = t.add("final", (item_id, j), yf[j])
    t = t.add("mean_z", 0, yf[2] / 1048576.0)
    return t, k


def photon(t, key, mu_a, mu_s):
    """benchmark configuration 3's item as a tallymap user writes it (csrc/items_photon.cuh states the same source):
    a photon random-walking through a 64^3 slab, Henyey-Greenstein scattering (g = 0.9), roulette below 1e-3"""
    g = 0.9
    mu_t = mu_a + mu_s
    albedo, frac = mu_s / mu_t, mu_a / mu_t

    def body(c):
        k, px, py, pz, dx, dy, dz, w, alive, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k), (4,))
        s = (-tl.log(1.0 - u[0])) / mu_t
        px, py, pz = px + s * dx, py + s * dy, pz + s * dz
        inside = (px >= 0.0) & (px < 64.0) & (py >= 0.0) & (py < 64.0) & (pz >= 0.0) & (pz < 64.0)
        ix, iy, iz = (tl.clip(q.astype(tl.int32), 0, 63) for q in (px, py, pz))
        t = t.add("dep", (ix, iy, iz), tl.where(inside, w * frac, 0.0))
        w1 = w * albedo
        tmp = (1 - g * g) / ((1 - g) + (2 * g) * u[1])
        cos_t = tl.clip(((1 + g * g) - tmp * tmp) / (2 * g), -1.0, 1.0)
        sin_t = tl.sqrt(1.0 - cos_t * cos_t)
        phi = (2 * 3.141592653589793) * u[2]
        sp, cp = tl.sin(phi), tl.cos(phi)
        r = tl.sqrt(1.0 - dz * dz)
        polar = tl.abs(dz) > 0.99999
        ndx = tl.where(polar, sin_t * cp, (sin_t * ((dx * dz) * cp - dy * sp)) / r + dx * cos_t)
        ndy = tl.where(polar, sin_t * sp, (sin_t * ((dy * dz) * cp + dx * sp)) / r + dy * cos_t)
        ndz = tl.where(polar, cos_t * tl.where(dz > 0.0, 1.0, -1.0), ((-sin_t) * cp) * r + dz * cos_t)
        low, survive = w1 < 1e-3, u[3] < 0.1
        w = tl.where(low, tl.where(survive, w1 * 10.0, 0.0), w1)
        return k + 1, px, py, pz, ndx, ndy, ndz, w, inside & ~(low & ~survive), t
    c = tl.while_loop(lambda c: c[8], body, (0, 32.0, 32.0, 0.0, 0.0, 0.0, 1.0, 1.0, True, t))
    return c[9], c[0]


def branch_writes(t, x, key, a):
    """tally writes inside lax.cond / lax.switch branches, made by the taken branch only (the reference threads the
    tally through lax.switch, tallymap/_rewrite.py:573-598): per step a switch on a draw adds to bin 0, to bin 1 or,
    in its last branch, appends a record through a nested cond when x < 0.25; a cond adds a * x to bin 3 above a
    half and 1 to bin 2 below; after the loop, bin 4 takes x when the walk ran its 40 steps"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        j = (u * 3.0).astype(tl.int32)
        t = tl.switch(j, [lambda tt: tt.add("h", 0, x * a),
                          lambda tt: tt.add("h", 1, a * a),
                          lambda tt: tl.cond(x < 0.25, lambda t2: t2.append("low", {"k": k, "x": x}),
                                             lambda t2: t2, tt)], t)
        t = tl.cond(x > 0.5, lambda tt: tt.add("h", 3, a * x), lambda tt: tt.add("h", 2, 1.0), t)
        return k + 1, x + 0.05 * (2.0 * u - 1.0), t
    k, x, t = tl.while_loop(lambda c: (c[0] < 40) & (c[1] >= 0.0) & (c[1] <= 1.0), body, (0, x, t))
    t = tl.cond(k == 40, lambda tt: tt.add("h", 4, x), lambda tt: tt, t)
    return t, k


def branch_writes_where(t, x, key, a):
    """branch_writes written without branches: each write at its bin every step, its value selected to zero (and a
    record's `when`) where the branch is not taken -- the same sums, records and gradients"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        j = tl.clip((u * 3.0).astype(tl.int32), 0, 2)
        t = t.add("h", 0, tl.where(j == 0, x * a, 0.0))
        t = t.add("h", 1, tl.where(j == 1, a * a, 0.0))
        t = t.append("low", {"k": k, "x": x}, when=(j == 2) & (x < 0.25))
        t = t.add("h", 3, tl.where(x > 0.5, a * x, 0.0))
        t = t.add("h", 2, tl.where(x > 0.5, 0.0, 1.0))
        return k + 1, x + 0.05 * (2.0 * u - 1.0), t
    k, x, t = tl.while_loop(lambda c: (c[0] < 40) & (c[1] >= 0.0) & (c[1] <= 1.0), body, (0, x, t))
    t = t.add("h", 4, tl.where(k == 40, x, 0.0))
    return t, k


def spawn_decay_cond(t, g, w, key, a):
    """spawn_decay with its child spawned from inside a lax.cond branch instead of by `when`"""
    def body(c):
        k, w, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        t = t.add("Q", k % 8, a * w * u)
        return k + 1, w * 0.9, t
    k, w, t = tl.while_loop(lambda c: c[0] < 3, body, (0, w, t))
    t = tl.cond(g < 2, lambda tt: tt.spawn((g + 1, w * a, tl.random.fold_in(key, 7))), lambda tt: tt, t)
    return t, k


def quickstart_hits(t, x, key, theta):
    """the quickstart walker appending {"x": x} at each step that starts in bin 3 (a Records output "hits")"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        b = (x * 16).astype(tl.int32)
        t = t.add("hist", b, theta * (1 - x))
        t = t.append("hits", {"x": x}, when=b == 3)
        return k + 1, x * (0.5 + 0.5 * u), t
    k, x, t = tl.while_loop(lambda c: c[1] > 0.05, body, (0, x, t))
    return t, k


def rejection(t, x, key, a):
    """inner while loops (the reference's C while, backends/kernel/op_table.py:1414-1450): each step of the walk
    draws (u, v) until u^2 + v^2 < 1 (at most 64 tries, a try counted into the int tally inside the inner loop,
    reading the step's key from outside it) and moves by 0.05 u; a step that starts above a half runs three more
    inner iterations in a cond branch; after the stepping loop, a second loop halves |x| while above 0.01 and a
    fori_loop with a traced bound sums 0..k%5-1"""
    def body(c):
        k, x, t = c
        kk = tl.random.fold_in(key, k)

        def draw(d):
            j, u, v, t = d
            kj = tl.random.fold_in(kk, j)
            u = 2.0 * tl.random.uniform(tl.random.fold_in(kj, 0)) - 1.0
            v = 2.0 * tl.random.uniform(tl.random.fold_in(kj, 1)) - 1.0
            return j + 1, u, v, t.add("tries", 0, 1)
        j, u, v, t = tl.while_loop(lambda d: (d[0] < 64) & (d[1] * d[1] + d[2] * d[2] >= 1.0), draw,
                                   (0, 1.0, 1.0, t))
        three = lambda tt: tl.while_loop(lambda d: d[0] < 3, lambda d: (d[0] + 1, d[1].add("tries", 1, 1)), (0, tt))[1]
        t = tl.cond(x > 0.5, three, lambda tt: tt, t)
        x = x + 0.05 * u
        t = t.add("h", (x * 8).astype(tl.int32), a * x)
        return k + 1, x, t
    k, x, t = tl.while_loop(lambda c: (c[0] < 200) & (c[1] > 0.0) & (c[1] < 1.0), body, (0, x, t))
    n, y = tl.while_loop(lambda c: (c[0] < 32) & (c[1] > 0.01), lambda c: (c[0] + 1, c[1] * 0.5), (0, tl.abs(x)))
    t = t.add("h", 8, a * y)
    s = tl.fori_loop(0, k % 5, lambda i, c: c + i, 0)
    return t, k, n, s


def rejection_active(t, x, key, a):
    """an inner loop that reads the differentiated operand a: lowered forward, refused by reverse mode"""
    def body(c):
        k, x, t = c
        j, y = tl.while_loop(lambda d: (d[0] < 4) & (d[1] < 1.0), lambda d: (d[0] + 1, d[1] + a), (0, x))
        return k + 1, x + 0.1, t.add("h", 0, y)
    k, x, t = tl.while_loop(lambda c: c[0] < 5, body, (0, x, t))
    return t, k


def newton(t, x, key, a):
    """each step runs 3 + k % 4 fixed-point iterations y <- x + a sin(y) (an inner loop whose carry and body read the
    differentiated a and the step's x, adding a * y to bin 1 at every iterate), adds the result to bin 0 and moves
    x by 0.1 y: an active stepping carry and an active inner loop, smooth in a"""
    def body(c):
        k, x, t = c

        def it(d):
            j, y, t = d
            y2 = x + a * tl.sin(y)
            return j + 1, y2, t.add("h", 1, a * y2)
        j, y, t = tl.while_loop(lambda d: d[0] < 3 + k % 4, it, (0, x, t))
        return k + 1, x + 0.1 * y, t.add("h", 0, y)
    k, x, t = tl.while_loop(lambda c: c[0] < 6, body, (0, x, t))
    return t, k


def loop_records(t, x, key, a):
    """Records appended inside inner loops: each step iterates y <- 0.5 y + x for 1 + k % 3 iterations, appending
    {"v": a y} at each (a loop that reads the differentiated a: its appends are transposed iteration by iteration),
    then a loop that reads no differentiated value appends {"v": x} twice (no cotangent, but it moves the append
    ordinal), and adds a y to the Sum"""
    def body(c):
        k, x, t = c

        def it(d):
            j, y, t = d
            y = 0.5 * y + x
            return j + 1, y, t.append("r", {"v": a * y})
        j, y, t = tl.while_loop(lambda d: d[0] < 1 + k % 3, it, (0, x, t))
        j2, t = tl.while_loop(lambda d: d[0] < 2, lambda d: (d[0] + 1, d[1].append("r", {"v": x})), (0, t))
        return k + 1, x + 0.1, t.add("h", 0, a * y)
    k, x, t = tl.while_loop(lambda c: c[0] < 4, body, (0, x, t))
    return t, k


def accumulators(t, x, key, a):
    """the wider accumulators (tallymap.Sum of float64, int64, and fixed_point with a scale): per step a drawn bin
    b of 4 takes a float v = 1000 a (u - 0.5) into a float64 Sum and a scaled float64 one, 1 + k into an int64 Sum,
    an int in [-50, 50) into a scaled int32 one, and the positive 500 a u into a float64 Sum at scale 2^50, whose
    words carry past 2^63 many times"""
    def body(c):
        k, x, t = c
        u = tl.random.uniform(tl.random.fold_in(key, k))
        b = (u * 4).astype(tl.int32)
        v = a * (u - 0.5) * 1000.0
        t = t.add("f64", b, v).add("i64", b, 1 + k).add("w64", b, v)
        t = t.add("wi32", b, (u * 100).astype(tl.int32) - 50).add("wbig", b, a * u * 500.0)
        return k + 1, x + 0.05 * (2 * u - 1), t
    k, x, t = tl.while_loop(lambda c: (c[1] >= 0) & (c[1] <= 1) & (c[0] < 100), body, (0, x, t))
    return t, k
