// Body-pair contacts: minimum portal refinement on inflated convex shapes.
// Included inside Solver<R, T> (solver.cuh).  Each lane runs the narrow phase
// of one collision pair on its own (the reference walks one portal with the
// whole warp and only shares the support-point search, convex.cuh:18-41);
// every operation uses the exact x-prefixed arithmetic so the result equals
// the reference's host build bit for bit (convex.cuh:9-217,
// kernel.cuh:654-722).

struct Sup { V3<R> v, a, b; };
struct Hit { int status; V3<R> normal, position; R depth; };

__device__ V3<R> xsupport(int s, int body, V3<R> d, R inflation) const {
  const Q4<R> q = quat(body);
  const V3<R> x = ld3(L.X + 3 * body);
  V3<R> ldir = xrotate(conj(q), d), local;
  const int type = ldg(m->sType[s]);
  if (type == 0 || type == 2) {
    V3<R> size = mv3(m->sSize[s]);
    local = xadd(mv3(m->sCenter[s]), xscale(xunit(ldir), size.x));
    if (type == 2) {
      V3<R> axis = xrotate(mq4(m->sQ[s]), V3<R>{R(0), R(0), R(1)});
      local = xadd(local, xscale(axis, xdot(axis, ldir) >= R(0) ? size.y : -size.y));
    }
  } else {
    const int offset = ldg(m->sOffset[s]), count = ldg(m->sCount[s]);
    int best = 0;
    R value = R(-INFINITY);
    for (int i = 0; i < count; ++i) {
      const R *p = pts + 3 * (offset + i);
      R c = xdot(V3<R>{ldg(p[0]), ldg(p[1]), ldg(p[2])}, ldir);
      if (c > value) { best = i; value = c; }
    }
    const R *p = pts + 3 * (offset + best);
    local = {ldg(p[0]), ldg(p[1]), ldg(p[2])};
  }
  return xadd(xadd(x, xrotate(q, local)), xscale(d, inflation));
}
__device__ Sup xminkowski(int sa, int ba, int sb, int bb, R inflation, V3<R> d) const {
  Sup p;
  p.a = xsupport(sa, ba, d, inflation / R(2));
  p.b = xsupport(sb, bb, -d, inflation / R(2));
  p.v = xsub(p.a, p.b);
  return p;
}
static __device__ V3<R> xportalDirection(const Sup *p) {
  return xunit(xcross(xsub(p[2].v, p[1].v), xsub(p[3].v, p[1].v)));
}
static __device__ void xexpandPortal(Sup *p, const Sup &v) {
  V3<R> c = xcross(v.v, p[0].v);
  if (xdot(p[1].v, c) > R(0)) {
    if (xdot(p[2].v, c) > R(0)) p[1] = v; else p[3] = v;
  } else if (xdot(p[3].v, c) > R(0)) {
    p[2] = v;
  } else {
    p[1] = v;
  }
}
static __device__ R xportalAdvance(const Sup *p, const Sup &v, V3<R> d) {
  return xsub(xdot(v.v, d), rmax(xdot(p[1].v, d), rmax(xdot(p[2].v, d), xdot(p[3].v, d))));
}
static __device__ V3<R> xclosestTriangle(V3<R> a, V3<R> b, V3<R> c) {
  V3<R> best = a;
  R distance = xdot(a, a);
  V3<R> v[3] = {a, b, c};
  for (int i = 0; i < 3; ++i) {
    V3<R> start = v[i], edge = xsub(v[(i + 1) % 3], start);
    R square = xdot(edge, edge);
    V3<R> point = xadd(start, xscale(edge, square > R(0) ? rclamp(-xdot(start, edge) / square, R(0), R(1)) : R(0)));
    if (xdot(point, point) < distance) {
      distance = xdot(point, point);
      best = point;
    }
  }
  V3<R> n = xcross(xsub(b, a), xsub(c, a));
  R nn = xdot(n, n);
  if (nn > R(0)) {
    V3<R> point = xscale(n, xdot(n, a) / nn);
    R u = xdot(xcross(xsub(b, point), xsub(c, point)), n) / nn;
    R w = xdot(xcross(xsub(c, point), xsub(a, point)), n) / nn;
    if (u >= R(0) && w >= R(0) && xadd(u, w) <= R(1) && xdot(point, point) < distance) best = point;
  }
  return best;
}
static __device__ V3<R> xportalPosition(const Sup *p, V3<R> d) {
  R w[4] = {xdot(xcross(p[1].v, p[2].v), p[3].v), xdot(xcross(p[3].v, p[2].v), p[0].v),
            xdot(xcross(p[0].v, p[1].v), p[3].v), xdot(xcross(p[2].v, p[1].v), p[0].v)};
  R sum = xadd(xadd(xadd(w[0], w[1]), w[2]), w[3]);
  if (!(sum > R(0))) {
    w[0] = R(0);
    w[1] = xdot(xcross(p[2].v, p[3].v), d);
    w[2] = xdot(xcross(p[3].v, p[1].v), d);
    w[3] = xdot(xcross(p[1].v, p[2].v), d);
    sum = xadd(xadd(w[1], w[2]), w[3]);
  }
  if (!(sum > R(0))) return {R(NAN), R(NAN), R(NAN)};
  V3<R> position{R(0), R(0), R(0)};
  for (int i = 0; i < 4; ++i) position = xadd(position, xscale(xadd(p[i].a, p[i].b), w[i] / xmul(R(2), sum)));
  return position;
}
// convexContact (convex.cuh:124-217) with bounded iterations: status 0
// separated, 1 intersecting, -1 indeterminate.
__device__ __forceinline__ Hit xconvexContact(int sa, int sb, R inflation, R tolerance) const {
  Hit result{0, {R(0), R(0), R(0)}, {R(0), R(0), R(0)}, R(0)};
  const int ba = ldg(m->sBody[sa]), bb = ldg(m->sBody[sb]);
  Sup p[4];
  p[0].a = xadd(ld3(L.X + 3 * ba), xrotate(quat(ba), mv3(m->sInterior[sa])));
  p[0].b = xadd(ld3(L.X + 3 * bb), xrotate(quat(bb), mv3(m->sInterior[sb])));
  p[0].v = xsub(p[0].a, p[0].b);
  const R scale = rmax(R(.001), xadd(ldg(m->sRadius[sa]), ldg(m->sRadius[sb])));
  const R epsilon = xmul(tolerance, R(.01));
  const R portalEps = xmul(xmul(-epsilon, scale), scale);
  if (xnorm(p[0].v) < epsilon) p[0].v.x = xadd(p[0].v.x, xmul(epsilon, R(10)));
  V3<R> d = xunit(-p[0].v);
  p[1] = xminkowski(sa, ba, sb, bb, inflation, d);
  if (xdot(p[1].v, d) <= R(0)) return result;
  d = xcross(p[0].v, p[1].v);
  if (xnorm(d) <= xmul(epsilon, scale)) {
    result.status = 1;
    result.depth = xnorm(p[1].v);
    result.normal = result.depth > epsilon ? -xunit(p[1].v) : xunit(p[0].v);
    result.position = xdiv(xadd(p[1].a, p[1].b), R(2));
    return result;
  }
  d = xunit(d);
  p[2] = xminkowski(sa, ba, sb, bb, inflation, d);
  if (xdot(p[2].v, d) <= R(0)) return result;
  d = xunit(xcross(xsub(p[1].v, p[0].v), xsub(p[2].v, p[0].v)));
  if (xdot(d, p[0].v) > R(0)) {
    Sup tmp = p[1];
    p[1] = p[2];
    p[2] = tmp;
    d = -d;
  }
  bool discovered = false;
  for (int it = 0; it < 128; ++it) {
    if (!isfinite(d.x)) break;
    p[3] = xminkowski(sa, ba, sb, bb, inflation, d);
    if (xdot(p[3].v, d) <= R(0)) return result;
    if (xdot(xcross(p[1].v, p[3].v), p[0].v) < portalEps) p[2] = p[3];
    else if (xdot(xcross(p[3].v, p[2].v), p[0].v) < portalEps) p[1] = p[3];
    else { discovered = true; break; }
    d = xunit(xcross(xsub(p[1].v, p[0].v), xsub(p[2].v, p[0].v)));
  }
  if (!discovered) { result.status = -1; return result; }
  bool intersecting = false;
  for (int it = 0; it < 128; ++it) {
    d = xportalDirection(p);
    if (!isfinite(d.x)) break;
    if (xdot(d, p[1].v) >= -epsilon) { intersecting = true; break; }
    Sup point = xminkowski(sa, ba, sb, bb, inflation, d);
    if (xdot(point.v, d) < R(0) || xportalAdvance(p, point, d) <= tolerance) return result;
    xexpandPortal(p, point);
  }
  if (!intersecting) { result.status = -1; return result; }
  for (int it = 0; it < 256; ++it) {
    d = xportalDirection(p);
    if (!isfinite(d.x)) break;
    Sup point = xminkowski(sa, ba, sb, bb, inflation, d);
    if (xportalAdvance(p, point, d) <= tolerance) {
      V3<R> closest = xclosestTriangle(p[1].v, p[2].v, p[3].v);
      result.depth = xnorm(closest);
      result.normal = result.depth > epsilon ? xdiv(-closest, result.depth) : -d;
      result.position = xportalPosition(p, d);
      result.status = isfinite(result.position.x) ? 1 : -1;
      return result;
    }
    xexpandPortal(p, point);
  }
  result.status = -1;
  return result;
}

// Self-contact generation and warm start (kernel.cuh:654-722); returns the
// new contact count.  Contacts follow the ground contacts in pair order.
// Body-pair contacts run out of line on a by-value copy of the solver: the
// caller's solver object never has its address taken, so it stays in
// registers, and the narrow-phase code stays out of the hot instruction
// stream.
__device__ __forceinline__ int detectPairs(int base, int prevCount) { return pairPass(*this, base, prevCount); }
static __device__ __noinline__ int pairPass(Solver self, int base, int prevCount) {
  return self.detectPairsBody(base, prevCount);
}
__device__ __forceinline__ int detectPairsBody(int base, int prevCount) {
  const R dt = m->dt;
  const R tolerance = rmax(R(1e-8), xmul(m->tolerance, R(.1)));
  const R ag = xmul(m->alpha, m->gamma);
  const R *prev = rec + kRecHeader + kRecBody * m->nb + kRecJoint * m->nj;
  const int nGround = base;
  // Pass 1, one lane per pair: the bounding-sphere test with the velocity
  // skin (kernel.cuh:656-664).  The pairs that pass are the narrow phase's
  // candidates; they are listed in pair order in the free contact entries
  // from nGround on (pair index in the meta word, skin in the c0 word), which
  // the contacts written in pass 2 overtake only after they are read.
  int candidates = 0;
  for (int first = 0; first < m->np; first += T) {
    const int pi = first + team.lane;
    bool close = false;
    R skin = R(0);
    if (pi < m->np) {
      const int sa = ldg(m->pA[pi]), sb = ldg(m->pB[pi]);
      const int ba = ldg(m->sBody[sa]), bb = ldg(m->sBody[sb]);
      if (!(ldg(m->mass[ba]) == R(0) && ldg(m->mass[bb]) == R(0))) {
        const R radA = ldg(m->sRadius[sa]), radB = ldg(m->sRadius[sb]);
        skin = xadd(R(.003), xmul(dt, xadd(xadd(xnorm(xsub(vel(ba), vel(bb))), xmul(xnorm(omega(ba)), radA)),
                                             xmul(xnorm(omega(bb)), radB))));
        close = !(xnorm(xsub(ld3(L.X + 3 * ba), ld3(L.X + 3 * bb))) > xadd(xadd(radA, radB), skin));
      }
    }
    int total;
    const int at = nGround + candidates + team.scan(close ? 1 : 0, &total);
    if (close) {
      if (at < L.cap) {
        cmeta(at) = pi;
        contact(at)[cC0] = skin;
      } else {
        I[iFailed] = 1;
      }
    }
    candidates += total;
  }
  candidates = nGround + candidates <= L.cap ? candidates : L.cap - nGround;
  team.sync();
  // Pass 2: the narrow phase (MPR) over the candidates only, so a team's
  // rounds of the costly portal search follow the number of close pairs, not
  // where they sit in the pair list.  Hits keep pair order.
  for (int first = 0; first < candidates; first += T) {
    const int k = first + team.lane;
    Hit hit{0, {R(0), R(0), R(0)}, {R(0), R(0), R(0)}, R(0)};
    R skin = R(0);
    int pi = 0, sa = 0, sb = 0, ba = 0, bb = 0;
    if (k < candidates) {
      pi = cmeta(nGround + k);
      skin = contact(nGround + k)[cC0];
    }
    team.sync();   // every candidate of this round is read before contacts are written
    if (k < candidates) {
      sa = ldg(m->pA[pi]);
      sb = ldg(m->pB[pi]);
      ba = ldg(m->sBody[sa]);
      bb = ldg(m->sBody[sb]);
      hit = xconvexContact(sa, sb, skin, tolerance);
      if (hit.status < 0) I[iFailed] = 1;
    }
    const int found = hit.status == 1 ? 1 : 0;
    int total;
    const int slot = base + team.scan(found, &total);
    if (found) {
      if (slot >= L.cap) {
        I[iFailed] = 1;
      } else {
        const Q4<R> qa = quat(ba), qb = quat(bb);
        const V3<R> n = hit.normal;
        const V3<R> ax = fabs(n.x) < R(.8) ? V3<R>{R(1), R(0), R(0)} : V3<R>{R(0), R(1), R(0)};
        const V3<R> t1 = xunit(xcross(ax, n));
        const V3<R> t2 = xcross(n, t1);
        const R gap = xsub(skin, hit.depth);
        const V3<R> half = xscale(n, gap / R(2));
        const V3<R> local = xrotate(conj(qa), xsub(xadd(hit.position, half), ld3(L.X + 3 * ba)));
        const V3<R> localB = xrotate(conj(qb), xsub(xsub(hit.position, half), ld3(L.X + 3 * bb)));
        R lambda[3] = {R(0), R(0), R(0)}, penalty[3] = {R(1000), R(1000), R(1000)};
        for (int i = 0; i < prevCount; ++i) {
          const R *o = prev + kRecContact * i;
          if (int(o[1]) != sa || int(o[4]) != sb) continue;
          V3<R> on{o[21], o[22], o[23]};
          if (!(xdot(on, n) > R(.95))) continue;
          if (!(xnorm(xrotate(qa, xsub(V3<R>{o[6], o[7], o[8]}, local))) < R(.005))) continue;
          if (!(xnorm(xrotate(qb, xsub(V3<R>{o[12], o[13], o[14]}, localB))) < R(.005))) continue;
          V3<R> f = xadd(xadd(xscale(V3<R>{o[15], o[16], o[17]}, o[26]), xscale(V3<R>{o[18], o[19], o[20]}, o[27])),
                         xscale(on, o[28]));
          lambda[0] = xdot(f, t1);
          lambda[1] = xdot(f, t2);
          lambda[2] = xdot(f, n);
          penalty[0] = o[29]; penalty[1] = o[30]; penalty[2] = o[31];
          break;
        }
        SV c = contact(slot);
        cmeta(slot) = packMeta(ba, bb, sa, sb);
        cfeat(slot) = 0;
        c[cLocal] = local.x; c[cLocal + 1] = local.y; c[cLocal + 2] = local.z;
        c[cAnchor] = localB.x; c[cAnchor + 1] = localB.y; c[cAnchor + 2] = localB.z;
        c[cFriction] = ldg(m->pFriction[pi]);
        c[cC0] = rmin(gap, R(0));
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          c[cLambda + d] = xmul(lambda[d], ag);
          c[cPenalty + d] = rclamp(xmul(penalty[d], m->gamma), R(1000), R(1e9));
        }
        SV bs = S + (L.CB + 9 * (slot - nGround));
        bs[0] = t1.x; bs[1] = t1.y; bs[2] = t1.z;
        bs[3] = t2.x; bs[4] = t2.y; bs[5] = t2.z;
        bs[6] = n.x; bs[7] = n.y; bs[8] = n.z;
      }
    }
    base += total;
  }
  base = base < L.cap ? base : L.cap;
  team.sync();
  // Fresh colours for contacts joining two bodies of one colour, in list order.
  if (team.lane == 0) {
    int colorCount = I[iColors];
    for (int ci = nGround; ci < base; ++ci) {
      const int meta = cmeta(ci);
      const int a = metaBody(meta), b = metaOther(meta);
      if (ldg(m->mass[a]) > R(0) && ldg(m->mass[b]) > R(0) && I[L.colors + a] == I[L.colors + b])
        I[L.colors + b] = colorCount++;
    }
    I[iColors] = colorCount;
  }
  team.sync();
  return base;
}
