"""Synthetic LIBERO-style scenes compiled to the normalized model arrays.

The reference builds its device model from a CPU-MuJoCo ``mjModel``
(libero/libero/gpu/host/backends/cuda_fp32/model.py:62-219, ``prepare``), which
needs ``mujoco==3.16.0`` (requirements-cuda-fp32.txt).  MuJoCo is not installed
here, so this module plays the MuJoCo compiler's role for the synthetic scenes
the benchmark names: it emits the same normalized arrays directly, computing
the compile-time constants the engine reads the way MuJoCo's ``mj_setConst``
does (``body_invweight0``, ``dof_invweight0``, ``stat.meaninertia`` from the
mass matrix at ``qpos0``).  Every inertial is explicit, so the MJCF text that
``Scene.mjcf()`` returns compiles to the same model wherever MuJoCo exists.

Scene A (BASELINE config 0/1): a Franka-like 7-hinge arm with capsule links
(r = 0.06), a 2-slide parallel gripper, a ground plane and three free boxes.
Scene B (config 2): the same arm plus 12 free objects (4 boxes, 4 capsules,
2 spheres, 2 hulls); hull colliders need the convex GJK/EPA path and are not
built in this revision (``Scene.supported`` says which families are).
"""
from dataclasses import dataclass, field
import math

import numpy as np

FREE, BALL, SLIDE, HINGE = 0, 1, 2, 3
PLANE, SPHERE, CAPSULE, BOX, MESH = 0, 2, 3, 6, 7

# robosuite Panda defaults (robosuite 1.4 panda robot + PandaGripper models).
PANDA_INIT_QPOS = [0.0, math.pi / 16.0, 0.0, -math.pi / 2.0 - math.pi / 3.0,
                   0.0, math.pi - 0.2, math.pi / 4.0]
PANDA_RANGES = [(-2.8973, 2.8973), (-1.7628, 1.7628), (-2.8973, 2.8973),
                (-3.0718, -0.0698), (-2.8973, 2.8973), (-0.0175, 3.7525),
                (-2.8973, 2.8973)]
PANDA_TORQUE = [80.0, 80.0, 80.0, 80.0, 12.0, 12.0, 12.0]
PANDA_MASS = [2.74, 2.74, 2.38, 2.43, 3.5, 1.47, 0.45]
GRIPPER_INIT = [0.020833, -0.020833]

DEFAULT_SOLREF = (0.02, 1.0)
DEFAULT_SOLIMP = (0.9, 0.95, 0.001, 0.5, 2.0)
DEFAULT_FRICTION = (1.0, 0.005, 0.0001)


def quat_mul(a, b):
    w1, x1, y1, z1 = a
    w2, x2, y2, z2 = b
    return np.array([w1 * w2 - x1 * x2 - y1 * y2 - z1 * z2,
                     w1 * x2 + x1 * w2 + y1 * z2 - z1 * y2,
                     w1 * y2 - x1 * z2 + y1 * w2 + z1 * x2,
                     w1 * z2 + x1 * y2 - y1 * x2 + z1 * w2])


def quat_mat(q):
    w, x, y, z = q
    return np.array([[w * w + x * x - y * y - z * z, 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), w * w - x * x + y * y - z * z, 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), w * w - x * x - y * y + z * z]])


def mat_quat(r):
    """Rotation matrix -> unit quaternion (w first, w >= 0)."""
    t = np.trace(r)
    if t > 0:
        s = math.sqrt(t + 1.0) * 2
        q = [0.25 * s, (r[2, 1] - r[1, 2]) / s, (r[0, 2] - r[2, 0]) / s, (r[1, 0] - r[0, 1]) / s]
    elif r[0, 0] > r[1, 1] and r[0, 0] > r[2, 2]:
        s = math.sqrt(1.0 + r[0, 0] - r[1, 1] - r[2, 2]) * 2
        q = [(r[2, 1] - r[1, 2]) / s, 0.25 * s, (r[0, 1] + r[1, 0]) / s, (r[0, 2] + r[2, 0]) / s]
    elif r[1, 1] > r[2, 2]:
        s = math.sqrt(1.0 + r[1, 1] - r[0, 0] - r[2, 2]) * 2
        q = [(r[0, 2] - r[2, 0]) / s, (r[0, 1] + r[1, 0]) / s, 0.25 * s, (r[1, 2] + r[2, 1]) / s]
    else:
        s = math.sqrt(1.0 + r[2, 2] - r[0, 0] - r[1, 1]) * 2
        q = [(r[1, 0] - r[0, 1]) / s, (r[0, 2] + r[2, 0]) / s, (r[1, 2] + r[2, 1]) / s, 0.25 * s]
    q = np.array(q)
    q /= np.linalg.norm(q)
    return q if q[0] >= 0 else -q


def _qmul_b(a, b):
    """Quaternion products of two batches [W, 4] (w, x, y, z)."""
    aw, ax, ay, az = a[:, 0], a[:, 1], a[:, 2], a[:, 3]
    bw, bx, by, bz = b[:, 0], b[:, 1], b[:, 2], b[:, 3]
    return np.stack([aw * bw - ax * bx - ay * by - az * bz, aw * bx + ax * bw + ay * bz - az * by,
                     aw * by - ax * bz + ay * bw + az * bx, aw * bz + ax * by - ay * bx + az * bw], axis=1)


def _qrot_b(q, v):
    """A vector [3] (or batch [W, 3]) rotated by a batch of quaternions [W, 4]."""
    u, w = q[:, 1:], q[:, :1]
    v = np.broadcast_to(v, u.shape)
    return 2 * np.sum(u * v, axis=1, keepdims=True) * u + (w * w - np.sum(u * u, axis=1, keepdims=True)) * v + \
        2 * w * np.cross(u, v)


def axis_quat(axis, angle):
    axis = np.asarray(axis, float) / np.linalg.norm(axis)
    return np.r_[math.cos(angle / 2), axis * math.sin(angle / 2)]


def geom_inertia(kind, size, mass):
    """Principal inertia of a solid primitive about its centre (geom frame)."""
    if kind == BOX:
        a, b, c = 2 * np.asarray(size[:3])
        return mass / 12.0 * np.array([b * b + c * c, a * a + c * c, a * a + b * b])
    if kind == SPHERE:
        r = size[0]
        return np.full(3, 0.4 * mass * r * r)
    if kind == CAPSULE:
        r, hl = size[0], size[1]
        h = 2 * hl
        vcyl, vsph = math.pi * r * r * h, 4.0 / 3.0 * math.pi * r ** 3
        mc, ms = mass * vcyl / (vcyl + vsph), mass * vsph / (vcyl + vsph)
        ixx = mc * (h * h / 12 + r * r / 4) + ms * (0.4 * r * r + h * h / 4 + 3 * h * r / 8)
        izz = mc * r * r / 2 + ms * 0.4 * r * r
        return np.array([ixx, ixx, izz])
    raise ValueError('no inertia for geom type %d' % kind)


def convex_mesh(points):
    """Convex hull of a point cloud as a mesh about its volume centroid.

    Returns the hull vertices (shifted so the centroid is the origin), its
    triangular faces wound outward with their unit normals, the volume and the
    inertia tensor per unit density about the centroid (signed tetrahedra
    from the centroid; Tonon 2004 / Blow-Binstock moment formulas)."""
    from scipy.spatial import ConvexHull
    pts = np.asarray(points, float)
    hull = ConvexHull(pts)
    keep = np.array(sorted(set(hull.vertices.tolist())))
    remap = {int(v): k for k, v in enumerate(keep)}
    vert = pts[keep]
    faces = []
    inside = vert.mean(axis=0)
    for simplex in hull.simplices:
        a, b, c = (remap[int(v)] for v in simplex)
        n = np.cross(vert[b] - vert[a], vert[c] - vert[a])
        if np.dot(n, vert[a] - inside) < 0:
            b, c = c, b
        faces.append((a, b, c))
    # volume and centroid
    vol, cen = 0.0, np.zeros(3)
    for a, b, c in faces:
        v = np.dot(vert[a] - inside, np.cross(vert[b] - inside, vert[c] - inside)) / 6.0
        vol += v
        cen += v * (vert[a] + vert[b] + vert[c] + inside) / 4.0
    cen /= vol
    vert = vert - cen
    # second moments of the tetrahedra (origin, a, b, c): integral of x x^T
    cov = np.zeros((3, 3))
    for a, b, c in faces:
        A = np.stack([vert[a], vert[b], vert[c]], axis=1)
        detA = np.linalg.det(A)
        canon = np.full((3, 3), 1.0 / 120.0) + np.eye(3) * (1.0 / 120.0)
        cov += detA * A @ canon @ A.T
    inertia = np.trace(cov) * np.eye(3) - cov
    normals = []
    for a, b, c in faces:
        n = np.cross(vert[b] - vert[a], vert[c] - vert[a])
        normals.append(n / np.linalg.norm(n))
    return dict(vert=vert, faces=faces, normals=np.array(normals), volume=vol, inertia=inertia)


@dataclass
class Geom:
    name: str
    kind: int
    size: tuple
    pos: tuple = (0, 0, 0)
    quat: tuple = (1, 0, 0, 0)
    contype: int = 1
    conaffinity: int = 1
    condim: int = 3
    friction: tuple = DEFAULT_FRICTION
    margin: float = 0.0
    mass: float = 0.0
    rgba: str = '0.7 0.7 0.7 1'
    mesh: dict = None  # convex_mesh() output for MESH geoms


@dataclass
class Joint:
    name: str
    kind: int
    axis: tuple = (0, 0, 1)
    pos: tuple = (0, 0, 0)
    range: tuple = None
    damping: float = 0.0
    armature: float = 0.0
    frictionloss: float = 0.0


@dataclass
class Body:
    name: str
    parent: int
    pos: tuple = (0, 0, 0)
    quat: tuple = (1, 0, 0, 0)
    joints: list = field(default_factory=list)
    geoms: list = field(default_factory=list)
    sites: list = field(default_factory=list)
    mass: float = None  # None: sum of geom masses


class Scene:
    """Normalized model arrays of one synthetic scene (host, float64)."""

    def __init__(self, name, bodies, actuators, options, capacities, controller):
        self.name = name
        self.bodies = bodies
        self.actuators = actuators
        self.options = options
        self.capacities = capacities
        self.controller = controller
        self._compile()

    # ------------------------------------------------------------------ compile
    def _compile(self):
        B = self.bodies
        nb = len(B)
        ints, reals = {}, {}
        parent = np.array([b.parent for b in B], np.int32)
        depth = np.zeros(nb, np.int32)
        for b in range(1, nb):
            assert parent[b] < b, 'bodies must be in depth-first order'
            depth[b] = depth[parent[b]] + 1
        # joints / dofs / qpos
        jnt, dofs, qadr = [], [], 0
        body_jntadr, body_jntnum, body_dofadr, body_dofnum = [], [], [], []
        for bi, b in enumerate(B):
            body_jntadr.append(len(jnt) if b.joints else -1)
            body_jntnum.append(len(b.joints))
            body_dofadr.append(len(dofs) if b.joints else -1)
            nd = 0
            for j in b.joints:
                width = {FREE: 6, BALL: 3, SLIDE: 1, HINGE: 1}[j.kind]
                jnt.append(dict(j=j, body=bi, qposadr=qadr, dofadr=len(dofs)))
                for _ in range(width):
                    dofs.append(dict(body=bi, jnt=len(jnt) - 1, damping=j.damping,
                                     armature=j.armature, frictionloss=j.frictionloss))
                qadr += {FREE: 7, BALL: 4, SLIDE: 1, HINGE: 1}[j.kind]
                nd += width
            body_dofnum.append(nd)
        nv, nq, nj = len(dofs), qadr, len(jnt)
        # dof parents (MuJoCo: previous dof of the same body, else last dof of
        # the nearest ancestor body with dofs)
        dof_parent = np.full(nv, -1, np.int32)
        body_lastdof = np.full(nb, -1, np.int32)
        for bi in range(nb):
            inherited = body_lastdof[parent[bi]] if bi > 0 else -1
            if body_dofnum[bi]:
                first = body_dofadr[bi]
                for k in range(body_dofnum[bi]):
                    dof_parent[first + k] = inherited if k == 0 else first + k - 1
                body_lastdof[bi] = first + body_dofnum[bi] - 1
            else:
                body_lastdof[bi] = inherited
        # weld / root / tree ids
        weld = np.zeros(nb, np.int32)
        root = np.zeros(nb, np.int32)
        for bi in range(1, nb):
            weld[bi] = bi if body_jntnum[bi] else weld[parent[bi]]
            root[bi] = bi if parent[bi] == 0 else root[parent[bi]]
        tree_of_root, trees = {}, []
        body_tree = np.full(nb, -1, np.int32)
        for bi in range(1, nb):
            if body_dofnum[bi] == 0 and body_lastdof[bi] < 0:
                continue
            r = root[bi]
            if r not in tree_of_root:
                tree_of_root[r] = len(trees)
                trees.append([])
            body_tree[bi] = tree_of_root[r]
        dof_tree = np.array([body_tree[d['body']] for d in dofs], np.int32)
        ntree = len(trees)
        tree_dofadr = np.array([int(np.flatnonzero(dof_tree == t)[0]) for t in range(ntree)], np.int32)
        tree_dofnum = np.array([int(np.sum(dof_tree == t)) for t in range(ntree)], np.int32)
        for t in range(ntree):
            assert np.all(np.flatnonzero(dof_tree == t) == tree_dofadr[t] + np.arange(tree_dofnum[t]))
        tree_madr = np.r_[0, np.cumsum(tree_dofnum ** 2)[:-1]].astype(np.int32)
        nM = int(np.sum(tree_dofnum ** 2))
        tri_sizes = tree_dofnum * (tree_dofnum + 1) // 2   # packed lower-triangular factor blocks
        tree_padr = np.r_[0, np.cumsum(tri_sizes)[:-1]].astype(np.int32)
        nL = int(np.sum(tri_sizes))
        # source of each packed lower-triangle entry in the dense tree blocks
        tree_lsrc = np.concatenate([tree_madr[t] + np.array([a * n + j for a in range(n) for j in range(a + 1)],
                                                            np.int64)
                                    for t, n in enumerate(tree_dofnum)]).astype(np.int32)
        # subtree intervals (depth-first order => contiguous)
        subtree_end = np.arange(nb, dtype=np.int32) + 1
        for bi in range(nb - 1, 0, -1):
            subtree_end[parent[bi]] = max(subtree_end[parent[bi]], subtree_end[bi])
        order = np.argsort(depth, kind='stable').astype(np.int32)
        nlevel = int(depth.max()) + 1
        level_start = np.searchsorted(depth[order], np.arange(nlevel + 1)).astype(np.int32)
        # ancestor dof masks (MJWarp body_isdofancestor, model.py prepare)
        dofmask = np.zeros((nb, 4), np.uint32)
        for bi in range(nb):
            d = body_lastdof[bi]
            while d >= 0:
                dofmask[bi, d // 32] |= np.uint32(1 << (d % 32))
                d = dof_parent[d]
        # body inertials from geoms (explicit <inertial> in the MJCF)
        body_mass = np.zeros(nb)
        body_ipos = np.zeros((nb, 3))
        body_iquat = np.tile([1.0, 0, 0, 0], (nb, 1))
        body_inertia = np.zeros((nb, 3))
        for bi, b in enumerate(B):
            if bi == 0:
                continue
            masses = [g.mass for g in b.geoms if g.mass > 0]
            total = sum(masses)
            if total <= 0:
                continue
            com = sum(g.mass * np.asarray(g.pos, float) for g in b.geoms if g.mass > 0) / total
            tensor = np.zeros((3, 3))
            for g in b.geoms:
                if g.mass <= 0:
                    continue
                r = quat_mat(np.asarray(g.quat, float) / np.linalg.norm(g.quat))
                if g.kind == MESH:
                    local = g.mass / g.mesh['volume'] * g.mesh['inertia']
                else:
                    local = np.diag(geom_inertia(g.kind, g.size, g.mass))
                tensor += r @ local @ r.T
                d = np.asarray(g.pos, float) - com
                tensor += g.mass * (np.dot(d, d) * np.eye(3) - np.outer(d, d))
            vals, vecs = np.linalg.eigh(tensor)
            if np.linalg.det(vecs) < 0:
                vecs[:, 0] = -vecs[:, 0]
            body_mass[bi] = total
            body_ipos[bi] = com
            body_iquat[bi] = mat_quat(vecs)
            body_inertia[bi] = vals
        subtreemass = body_mass.copy()
        for bi in range(nb - 1, 0, -1):
            subtreemass[parent[bi]] += subtreemass[bi]
        # geoms
        G = [(bi, g) for bi, b in enumerate(B) for g in b.geoms]
        ng = len(G)
        gtype = np.array([g.kind for _, g in G], np.int32)
        gbody = np.array([bi for bi, _ in G], np.int32)
        gsize = np.array([list(g.size) + [0.0] * (3 - len(g.size)) for _, g in G], float)
        aabb = np.zeros((ng, 6))
        rbound = np.zeros(ng)
        for k, (_, g) in enumerate(G):
            s = gsize[k]
            if g.kind == BOX:
                aabb[k, 3:] = s
                rbound[k] = np.linalg.norm(s)
            elif g.kind == SPHERE:
                aabb[k, 3:] = s[0]
                rbound[k] = s[0]
            elif g.kind == CAPSULE:
                aabb[k, 3:] = [s[0], s[0], s[0] + s[1]]
                rbound[k] = s[0] + s[1]
            elif g.kind == PLANE:
                aabb[k, 3:] = [1e10, 1e10, 0.0]
                rbound[k] = 0.0
            elif g.kind == MESH:
                v = g.mesh['vert']
                lo, hi = v.min(axis=0), v.max(axis=0)
                aabb[k, :3], aabb[k, 3:] = (lo + hi) / 2, (hi - lo) / 2
                gsize[k] = (hi - lo) / 2
                rbound[k] = float(np.max(np.linalg.norm(v, axis=1)))
        # mesh data (geom_dataid; vertices, polygons and the vertex -> polygon map)
        dataid = np.full(ng, -1, np.int32)
        mesh_vertadr, mesh_vertnum, mesh_polyadr, mesh_polynum = [], [], [], []
        mesh_vert, polyvertadr, polyvertnum, polyvert, polynormal = [], [], [], [], []
        polymapadr, polymapnum, polymap = [], [], []
        for k, (_, g) in enumerate(G):
            if g.kind != MESH:
                continue
            dataid[k] = len(mesh_vertadr)
            v, faces = g.mesh['vert'], g.mesh['faces']
            mesh_vertadr.append(len(mesh_vert))
            mesh_vertnum.append(len(v))
            mesh_polyadr.append(len(polyvertadr))
            mesh_polynum.append(len(faces))
            incident = [[] for _ in range(len(v))]
            for f, face in enumerate(faces):
                polyvertadr.append(len(polyvert))
                polyvertnum.append(len(face))
                polyvert.extend(int(x) for x in face)
                polynormal.append(g.mesh['normals'][f])
                for x in face:
                    incident[x].append(f)
            for x in range(len(v)):
                polymapadr.append(len(polymap))
                polymapnum.append(len(incident[x]))
                polymap.extend(incident[x])
            mesh_vert.extend(v.tolist())
        # collision pair filter (cuda_fp32/model.py:171-186 prepare_collision)
        contype = np.array([g.contype for _, g in G], np.int64)
        conaff = np.array([g.conaffinity for _, g in G], np.int64)
        pairs = []
        for i in range(ng):
            for j in range(i + 1, ng):
                b1, b2 = gbody[i], gbody[j]
                w1, w2 = weld[b1], weld[b2]
                p1, p2 = weld[parent[w1]], weld[parent[w2]]
                if not ((contype[i] & conaff[j]) or (contype[j] & conaff[i])):
                    continue
                if w1 == w2:
                    continue
                if body_dofnum[w1] == 0 and body_dofnum[w2] == 0:
                    continue
                if w1 != 0 and w2 != 0 and (w1 == p2 or w2 == p1):
                    continue
                # broadphase emits the lower geom type first (mjwarp_broadphase.cu:112-113)
                pairs.append((j, i) if gtype[i] > gtype[j] else (i, j))
        self.pair_families = sorted({(int(gtype[a]), int(gtype[b])) for a, b in pairs})
        # box-box pairs take the convex path (GJK/EPA and the box manifold)
        # unless one of them has a margin (cuda_fp32/model.py:187-191,
        # physics.py:89-90); the per-pair margin there is the larger geom margin
        gmargin = np.array([g.margin for _, g in G], float)
        boxbox = [(a, b) for a, b in pairs if gtype[a] == BOX and gtype[b] == BOX]
        boxbox_convex = int(not any(max(gmargin[a], gmargin[b]) > 0 for a, b in boxbox))
        # MJWarp's EPA budget: 16 when every convex pair is box-box, else the CCD iterations
        convex_pairs = [(a, b) for a, b in pairs if gtype[b] == MESH and gtype[a] != PLANE] + \
            (boxbox if boxbox_convex else [])
        epa_default = 16 if convex_pairs and all(gtype[a] == BOX and gtype[b] == BOX for a, b in convex_pairs) \
            else self.options.get('ccd_iterations', 50)
        # sites
        S = [(bi, s) for bi, b in enumerate(B) for s in b.sites]
        ns = len(S)
        # limits / frictionloss
        limited = np.array([1 if j['j'].range is not None else 0 for j in jnt], np.int32)
        jrange = np.array([j['j'].range if j['j'].range is not None else (0.0, 0.0) for j in jnt], float)
        fric = np.array([d['frictionloss'] for d in dofs])
        # actuators
        A = self.actuators
        nu = len(A)
        # ---------------------------------------------------------------- pack
        qpos0 = np.zeros(nq)
        for j in jnt:
            if j['j'].kind == FREE:
                b = B[j['body']]
                qpos0[j['qposadr']:j['qposadr'] + 3] = b.pos
                qpos0[j['qposadr'] + 3:j['qposadr'] + 7] = b.quat
            elif j['j'].kind == BALL:
                qpos0[j['qposadr']:j['qposadr'] + 4] = [1, 0, 0, 0]
        opt = self.options
        cap = self.capacities
        self.sizes = dict(nq=nq, nv=nv, nu=nu, nbody=nb, njnt=nj, ngeom=ng, nsite=ns,
                          npair=len(pairs), ntree=ntree, nM=nM, nL=nL, nlevel=nlevel,
                          nlimited=int(limited.sum()), nfric=int(np.sum(fric > 0)),
                          nmesh=len(mesh_vertadr), nmeshvert=len(mesh_vert), nmeshpoly=len(polyvertadr),
                          nmeshpolyvert=len(polyvert), nmeshpolymap=len(polymap),
                          ccd_iterations=opt.get('ccd_iterations', 50),
                          epa_iterations=opt.get('epa_iterations', epa_default), boxbox_convex=boxbox_convex)
        ncon_max = cap['nconmax']
        cone = opt['cone']
        rows_per_contact = 3 if cone == 1 else 4
        nefc_max = cap.get('njmax') or (rows_per_contact * ncon_max + self.sizes['nlimited'] + self.sizes['nfric'])
        nvs = nv | 1  # odd row stride: conflict-free column walks in shared memory
        pair_dofs = [int(tree_dofnum[body_tree[gbody[a]]] if body_tree[gbody[a]] >= 0 else 0) +
                     int(tree_dofnum[body_tree[gbody[b]]] if body_tree[gbody[b]] >= 0 else 0)
                     for a, b in pairs]
        free_bodies = [j['body'] for j in jnt if j['j'].kind == FREE]
        self.sizes.update(nfree=len(free_bodies), nobs=9 + 9 + 3 + 4 + 7 * len(free_bodies) + 2)
        self.sizes.update(ncon_max=ncon_max, nefc_max=int(nefc_max), cone=cone,
                          iterations=opt['iterations'], ls_iterations=opt['ls_iterations'],
                          disable_flags=opt.get('disable_flags', 0),
                          ee_site=[s.name for _, s in S].index(self.controller['site']),
                          nvs=nvs, kmax_dof=max(pair_dofs + [1]), max_tree_dofs=int(tree_dofnum.max()),
                          osc_uncouple=int(self.controller.get('uncouple', True)),
                          task_body=int(opt.get('task_body', 0 if free_bodies else -1)))
        ints.update(
            body_parentid=parent, body_rootid=root, body_weldid=weld,
            body_jntnum=np.array(body_jntnum, np.int32), body_jntadr=np.array(body_jntadr, np.int32),
            body_dofnum=np.array(body_dofnum, np.int32), body_dofadr=np.array(body_dofadr, np.int32),
            body_treeid=body_tree, body_subtree_end=subtree_end, body_order=order,
            level_start=level_start, body_dofmask=dofmask.view(np.int32).reshape(-1),
            jnt_type=np.array([j['j'].kind for j in jnt], np.int32),
            jnt_qposadr=np.array([j['qposadr'] for j in jnt], np.int32),
            jnt_dofadr=np.array([j['dofadr'] for j in jnt], np.int32),
            jnt_bodyid=np.array([j['body'] for j in jnt], np.int32), jnt_limited=limited,
            dof_bodyid=np.array([d['body'] for d in dofs], np.int32),
            dof_jntid=np.array([d['jnt'] for d in dofs], np.int32),
            dof_parentid=dof_parent, dof_treeid=dof_tree,
            tree_dofadr=tree_dofadr, tree_dofnum=tree_dofnum, tree_madr=tree_madr, tree_padr=tree_padr,
            tree_lsrc=tree_lsrc,
            geom_type=gtype, geom_bodyid=gbody,
            geom_condim=np.array([g.condim for _, g in G], np.int32),
            geom_priority=np.zeros(ng, np.int32),
            site_bodyid=np.array([bi for bi, _ in S], np.int32),
            pair_geom=np.array(pairs, np.int32).reshape(-1),
            limited_jnt=np.flatnonzero(limited).astype(np.int32),
            fric_dof=np.flatnonzero(fric > 0).astype(np.int32),
            actuator_trnid=np.array([a['joint'] for a in A], np.int32),
            actuator_gaintype=np.array([a['gaintype'] for a in A], np.int32),
            actuator_biastype=np.array([a['biastype'] for a in A], np.int32),
            actuator_ctrllimited=np.array([1 if a.get('ctrlrange') else 0 for a in A], np.int32),
            actuator_forcelimited=np.array([1 if a.get('forcerange') else 0 for a in A], np.int32),
            osc_qposadr=np.array([jnt[k]['qposadr'] for k in self.controller['joints']], np.int32),
            osc_dofadr=np.array([jnt[k]['dofadr'] for k in self.controller['joints']], np.int32),
            osc_actuator=np.array(self.controller['actuators'], np.int32),
            free_bodyid=np.array(free_bodies, np.int32),
            geom_dataid=dataid, mesh_vertadr=np.array(mesh_vertadr, np.int32),
            mesh_vertnum=np.array(mesh_vertnum, np.int32), mesh_polyadr=np.array(mesh_polyadr, np.int32),
            mesh_polynum=np.array(mesh_polynum, np.int32), mesh_polyvertadr=np.array(polyvertadr, np.int32),
            mesh_polyvertnum=np.array(polyvertnum, np.int32), mesh_polyvert=np.array(polyvert, np.int32),
            mesh_polymapadr=np.array(polymapadr, np.int32), mesh_polymapnum=np.array(polymapnum, np.int32),
            mesh_polymap=np.array(polymap, np.int32))
        reals.update(
            body_pos=np.array([b.pos for b in B], float), body_quat=np.array([b.quat for b in B], float),
            body_ipos=body_ipos, body_iquat=body_iquat, body_mass=body_mass,
            body_subtreemass=subtreemass, body_inertia=body_inertia,
            jnt_pos=np.array([j['j'].pos for j in jnt], float), jnt_axis=np.array([j['j'].axis for j in jnt], float),
            jnt_range=jrange, jnt_margin=np.zeros(nj),
            jnt_solref=np.tile(DEFAULT_SOLREF, (nj, 1)), jnt_solimp=np.tile(DEFAULT_SOLIMP, (nj, 1)),
            jnt_stiffness=np.zeros(nj), qpos0=qpos0, qpos_spring=qpos0.copy(),
            dof_armature=np.array([d['armature'] for d in dofs]), dof_damping=np.array([d['damping'] for d in dofs]),
            dof_frictionloss=fric, dof_solref=np.tile(DEFAULT_SOLREF, (nv, 1)),
            dof_solimp=np.tile(DEFAULT_SOLIMP, (nv, 1)),
            geom_size=gsize, geom_pos=np.array([g.pos for _, g in G], float),
            geom_quat=np.array([g.quat for _, g in G], float), geom_aabb=aabb, geom_rbound=rbound,
            geom_friction=np.array([g.friction for _, g in G], float), geom_solmix=np.ones(ng),
            geom_solref=np.tile(DEFAULT_SOLREF, (ng, 1)), geom_solimp=np.tile(DEFAULT_SOLIMP, (ng, 1)),
            geom_margin=np.array([g.margin for _, g in G], float), geom_gap=np.zeros(ng),
            site_pos=np.array([s['pos'] for _, s in S], float).reshape(-1, 3),
            site_quat=np.array([s.get('quat', (1, 0, 0, 0)) for _, s in S], float).reshape(-1, 4),
            actuator_gear=np.array([a.get('gear', 1.0) for a in A], float),
            actuator_gainprm=np.array([a['gainprm'] for a in A], float),
            actuator_biasprm=np.array([a['biasprm'] for a in A], float),
            actuator_ctrlrange=np.array([a.get('ctrlrange') or (0, 0) for a in A], float),
            actuator_forcerange=np.array([a.get('forcerange') or (0, 0) for a in A], float),
            mesh_vert=np.array(mesh_vert, float).reshape(-1), mesh_polynormal=np.array(polynormal, float).reshape(-1))
        c = self.controller
        kp = np.broadcast_to(np.asarray(c['kp'], float), (6,))
        kd = 2 * np.sqrt(kp) * np.asarray(c.get('damping_ratio', 1.0))
        cfg = np.zeros(25)
        cfg[0:6], cfg[6:12] = -1.0, 1.0
        cfg[12:18] = [-0.05] * 3 + [-0.5] * 3
        cfg[18:24] = [0.05] * 3 + [0.5] * 3
        cfg[24] = 0.01
        reals.update(osc_gains=np.r_[kp, kd], osc_q0=np.asarray(c['q0'], float),
                     osc_action_config=cfg, osc_null=np.array([10.0, 2 * math.sqrt(10.0)]))
        self.ints, self.reals = ints, reals
        self.scalars = dict(timestep=opt['timestep'], gravity_x=0.0, gravity_y=0.0, gravity_z=-9.81,
                            tolerance=max(opt['tolerance'], 1e-6), ls_tolerance=opt.get('ls_tolerance', 0.01),
                            impratio_invsqrt=1.0 / math.sqrt(max(opt.get('impratio', 1.0), 1e-15)),
                            meaninertia=1.0, ccd_tolerance=opt.get('ccd_tolerance', 1e-6),
                            task_lift_z=opt.get('task_lift_z', 0.2))
        self.geom_names = [g.name for _, g in G]
        self.body_names = [b.name for b in B]
        self._set_const()

    # ------------------------------------------------------------- constants
    def _set_const(self):
        """MuJoCo mj_setConst: invweights and meaninertia at qpos0 (float64)."""
        from . import kinematics_host as kh
        state = kh.forward_position(self, self.reals['qpos0'])
        M = state['M_dense']
        Minv = np.linalg.inv(M)
        nv = self.sizes['nv']
        nb = self.sizes['nbody']
        self.scalars['meaninertia'] = float(np.mean(np.diag(M)))
        inv0 = np.zeros((nb, 2))
        for b in range(1, nb):
            if self.ints['body_weldid'][b] == 0:
                continue
            jp, jr = kh.body_jacobian(self, state, b, state['xipos'][b])
            inv0[b, 0] = np.trace(jp @ Minv @ jp.T) / 3.0
            inv0[b, 1] = np.trace(jr @ Minv @ jr.T) / 3.0
        self.reals['body_invweight0'] = np.maximum(inv0, 0.0)
        dofw = np.zeros(nv)
        for j, kind in enumerate(self.ints['jnt_type']):
            d = self.ints['jnt_dofadr'][j]
            if kind == FREE:
                dofw[d:d + 3] = np.mean(np.diag(Minv)[d:d + 3])
                dofw[d + 3:d + 6] = np.mean(np.diag(Minv)[d + 3:d + 6])
            elif kind == BALL:
                dofw[d:d + 3] = np.mean(np.diag(Minv)[d:d + 3])
            else:
                dofw[d] = Minv[d, d]
        self.reals['dof_invweight0'] = dofw

    # ---------------------------------------------------------------- states
    PLACEMENT_ATTEMPTS = 160
    CLEARANCE = 0.002      # object-object and object-floor gap at placement
    ARM_CLEARANCE = 0.005  # object-arm gap at placement

    def initial_state(self, nworld, seed=0, world_offset=0):
        """Per-world initial qpos/qvel, seeded per global world index.

        Worlds draw from ``SeedSequence(seed).spawn`` indexed by their global
        world number, so a shard's worlds do not depend on the GPU count.  A
        world's arm joints are its nominal pose plus N(0, 0.05^2) noise; its
        objects are then placed one after another by rejection sampling, each
        candidate drawn from the world's own stream, so that no object starts
        inside the floor, another object or any arm collision geom (the arm
        taken at that world's own joint angles).  Dropped objects fall from a
        centre height U[0.05, 0.15] m, raised where needed until their
        bounding sphere clears the floor."""
        nq, nv = self.sizes['nq'], self.sizes['nv']
        qpos = np.tile(self.reals['qpos0'], (nworld, 1))
        children = np.random.SeedSequence(seed).spawn(world_offset + nworld)[world_offset:]
        rngs = [np.random.default_rng(child) for child in children]
        c = self.controller
        adr = self.ints['jnt_qposadr']
        noise = np.stack([r.normal(0.0, 0.05, len(c['joints'])) for r in rngs]) if nworld else np.zeros((0, 7))
        for k, j in enumerate(c['joints']):
            qpos[:, adr[j]] = c['q0'][k] + noise[:, k]
        for j, value in zip(c['gripper_joints'], GRIPPER_INIT):
            qpos[:, adr[j]] = value
        nobj = len(self.objects)
        if nworld and nobj:
            draws = np.stack([r.random((nobj, self.PLACEMENT_ATTEMPTS, 6)) for r in rngs])
            for a in range(0, nworld, 4096):
                self._place_objects(qpos[a:a + 4096], draws[a:a + 4096])
        return qpos, np.zeros((nworld, nv))

    def _arm_segments(self, qpos):
        """Collision geoms of the non-free bodies (arm, hand, fingers) as
        capsule segments (p0, p1, radius) in world frame, for a batch of
        states: [W, ngeom_arm, 2, 3] end points and [ngeom_arm] radii (boxes
        and spheres as zero-length segments of their bounding radius)."""
        I, R = self.ints, self.reals
        W, nb = len(qpos), self.sizes['nbody']
        xpos = np.zeros((W, nb, 3))
        xquat = np.zeros((W, nb, 4))
        xquat[:, 0, 0] = 1
        free = np.zeros(nb, bool)
        for b in range(1, nb):
            first, count = I['body_jntadr'][b], I['body_jntnum'][b]
            if count == 1 and I['jnt_type'][first] == FREE:
                free[b] = True
                continue
            p = I['body_parentid'][b]
            pos = _qrot_b(xquat[:, p], R['body_pos'][b]) + xpos[:, p]
            quat = _qmul_b(xquat[:, p], np.broadcast_to(R['body_quat'][b], (W, 4)))
            for j in range(first, first + count):
                a, kind = I['jnt_qposadr'][j], I['jnt_type'][j]
                lpos, lax = R['jnt_pos'][j], R['jnt_axis'][j]
                anchor = _qrot_b(quat, lpos) + pos
                if kind == SLIDE:
                    pos = pos + _qrot_b(quat, lax) * (qpos[:, a] - R['qpos0'][a])[:, None]
                elif kind == HINGE:
                    half = 0.5 * (qpos[:, a] - R['qpos0'][a])
                    rq = np.concatenate([np.cos(half)[:, None], np.sin(half)[:, None] * lax], axis=1)
                    quat = _qmul_b(quat, rq)
                    pos = anchor - _qrot_b(quat, lpos)
            xpos[:, b], xquat[:, b] = pos, quat
        segs, radii = [], []
        for g in range(self.sizes['ngeom']):
            b = I['geom_bodyid'][g]
            if b == 0 or free[b]:
                continue
            kind, size = I['geom_type'][g], np.reshape(R['geom_size'], (-1, 3))[g]
            centre = _qrot_b(xquat[:, b], np.reshape(R['geom_pos'], (-1, 3))[g]) + xpos[:, b]
            if kind == CAPSULE:
                gq = _qmul_b(xquat[:, b], np.broadcast_to(np.reshape(R['geom_quat'], (-1, 4))[g], (W, 4)))
                axis = _qrot_b(gq, np.array([0.0, 0.0, 1.0])) * size[1]
                segs.append(np.stack([centre - axis, centre + axis], axis=1))
                radii.append(size[0])
            else:
                segs.append(np.stack([centre, centre], axis=1))
                radii.append(float(np.linalg.norm(size)) if kind == BOX else size[0])
        return np.stack(segs, axis=1), np.array(radii)

    def _place_objects(self, qpos, draws):
        """Rejection placement of the free objects for a batch of worlds;
        draws[w, object, attempt] holds six uniforms of world w's stream.  A
        world takes its first candidate that clears everything, else (all
        candidates failing) the one with the smallest overlap; candidates are
        examined in blocks, each block only for the worlds still looking."""
        W, A = len(qpos), draws.shape[2]
        segs, radii = self._arm_segments(qpos)
        p0, d = segs[:, :, 0], segs[:, :, 1] - segs[:, :, 0]          # [W, S, 3]
        dd = np.maximum(np.einsum('wsk,wsk->ws', d, d), 1e-30)
        placed = []  # (centre [W, 3], radius)
        for k, body in enumerate(self.objects):
            rbound = body.get('rbound', body['radius'])

            def candidates(u):
                xy = (u[..., 0:2] - 0.5) * self.object_square + self.object_center
                if body['drop'] is None:
                    z = np.full(u.shape[:-1], body['rest_z'])
                else:
                    lo, hi = body['drop']
                    z = np.maximum(lo + (hi - lo) * u[..., 2], rbound + self.CLEARANCE)
                return np.concatenate([xy, z[..., None]], axis=-1)

            def overlap(ws, cand):  # worst violation of each candidate of worlds ws
                short = np.full(cand.shape[:2], -np.inf)
                for centre, r in placed:
                    dist = np.linalg.norm(cand - centre[ws, None], axis=-1)
                    short = np.maximum(short, body['radius'] + r + self.CLEARANCE - dist)
                rel = cand[:, :, None, :] - p0[ws, None]
                tt = np.clip(np.einsum('wask,wsk->was', rel, d[ws]) / dd[ws, None], 0.0, 1.0)
                arm = np.linalg.norm(rel - tt[..., None] * d[ws, None], axis=-1)
                return np.maximum(short, np.max(rbound + radii + self.ARM_CLEARANCE - arm, axis=-1))

            pick = np.full(W, -1)
            best = np.full(W, np.inf)
            fallback = np.zeros(W, int)
            pending = np.arange(W)
            for a0 in range(0, A, 16):
                if not len(pending):
                    break
                short = overlap(pending, candidates(draws[pending, k, a0:a0 + 16]))
                ok = short <= 0
                hit = ok.any(axis=1)
                pick[pending[hit]] = a0 + ok[hit].argmax(axis=1)
                low = short.min(axis=1)
                better = low < best[pending]
                fallback[pending[better]] = a0 + short[better].argmin(axis=1)
                best[pending[better]] = low[better]
                pending = pending[~hit]
            pick[pending] = fallback[pending]
            ua = draws[np.arange(W), k, pick]
            centre = candidates(ua[:, None])[:, 0]
            placed.append((centre, body['radius']))
            a = self.ints['jnt_qposadr'][self.ints['body_jntadr'][body['id']]]
            qpos[:, a:a + 3] = centre
            if body.get('tumble'):  # dropped objects: uniformly random orientation (Shoemake)
                s1, s2 = np.sqrt(1.0 - ua[:, 3]), np.sqrt(ua[:, 3])
                th1, th2 = 2 * math.pi * ua[:, 4], 2 * math.pi * ua[:, 5]
                qpos[:, a + 3:a + 7] = np.stack([s2 * np.cos(th2), s1 * np.sin(th1), s1 * np.cos(th1),
                                                 s2 * np.sin(th2)], axis=1)
            else:
                yaw = (2 * ua[:, 3] - 1) * math.pi
                qpos[:, a + 3:a + 7] = np.stack([np.cos(yaw / 2), 0 * yaw, 0 * yaw, np.sin(yaw / 2)], axis=1)

    def actions(self, nworld, step, seed=0, world_offset=0):
        """Seeded OSC_POSE actions: U[-1,1]^6 plus a gripper sign in {-1,1}.

        Drawn per global world index (one stream per step, the first
        world_offset + nworld draws), so a shard's actions do not depend on
        the GPU count."""
        n = world_offset + nworld
        a = np.random.default_rng([seed, 7919, step, 0]).uniform(-1.0, 1.0, (n, 7))[world_offset:]
        grip = np.random.default_rng([seed, 7919, step, 1]).uniform(size=n)[world_offset:]
        a[:, 6] = np.where(grip < 0.5, -1.0, 1.0)
        return a

    @property
    def supported(self):
        known = {(PLANE, SPHERE), (PLANE, CAPSULE), (PLANE, BOX), (PLANE, MESH), (SPHERE, BOX),
                 (CAPSULE, BOX), (BOX, BOX), (SPHERE, SPHERE), (SPHERE, CAPSULE),
                 (CAPSULE, CAPSULE), (SPHERE, MESH), (CAPSULE, MESH), (BOX, MESH), (MESH, MESH)}
        return all(f in known for f in self.pair_families)

    # ------------------------------------------------------------------ mjcf
    def mjcf(self):
        """MJCF text of this scene (explicit inertials; compiles in MuJoCo)."""
        names = {PLANE: 'plane', SPHERE: 'sphere', CAPSULE: 'capsule', BOX: 'box', MESH: 'mesh'}
        kinds = {FREE: 'free', BALL: 'ball', SLIDE: 'slide', HINGE: 'hinge'}
        o = self.options
        out = ['<mujoco model="%s">' % self.name,
               '  <option timestep="%g" iterations="%d" ls_iterations="%d" tolerance="%g" '
               'cone="%s" impratio="%g" solver="Newton" integrator="Euler" jacobian="dense"/>' % (
                   o['timestep'], o['iterations'], o['ls_iterations'], o['tolerance'],
                   'elliptic' if o['cone'] == 1 else 'pyramidal', o.get('impratio', 1.0)),
               ]
        meshes = [g for b in self.bodies for g in b.geoms if g.kind == MESH]
        if meshes:
            out.append('  <asset>')
            for g in meshes:
                out.append('    <mesh name="%s_mesh" vertex="%s"/>' % (
                    g.name, ' '.join('%.9g' % v for v in g.mesh['vert'].reshape(-1))))
            out.append('  </asset>')
        out.append('  <worldbody>')
        depth = {0: 1}
        stack = [0]
        r = self.reals
        for bi, b in enumerate(self.bodies):
            if bi > 0:
                while stack[-1] != b.parent:
                    stack.pop()
                    out.append('  ' * depth[stack[-1] if stack else 0] + '  </body>')
                ind = '  ' * (depth[b.parent] + 1)
                depth[bi] = depth[b.parent] + 1
                out.append(ind + '<body name="%s" pos="%s" quat="%s">' % (
                    b.name, ' '.join('%.9g' % v for v in b.pos), ' '.join('%.9g' % v for v in b.quat)))
                if r['body_mass'][bi] > 0:
                    out.append(ind + '  <inertial pos="%s" quat="%s" mass="%.9g" diaginertia="%s"/>' % (
                        ' '.join('%.9g' % v for v in r['body_ipos'][bi]),
                        ' '.join('%.9g' % v for v in r['body_iquat'][bi]), r['body_mass'][bi],
                        ' '.join('%.9g' % v for v in r['body_inertia'][bi])))
                stack.append(bi)
            ind = '  ' * (depth[bi] + 1)
            for j in b.joints:
                s = '<joint name="%s" type="%s"' % (j.name, kinds[j.kind])
                if j.kind != FREE:
                    s += ' axis="%s" pos="%s"' % (' '.join('%g' % v for v in j.axis), ' '.join('%g' % v for v in j.pos))
                if j.range is not None:
                    s += ' limited="true" range="%.9g %.9g"' % j.range
                s += ' damping="%g" armature="%g" frictionloss="%g"/>' % (j.damping, j.armature, j.frictionloss)
                out.append(ind + s)
            for g in b.geoms:
                out.append(ind + '<geom name="%s" type="%s" %s pos="%s" quat="%s" contype="%d" '
                           'conaffinity="%d" condim="%d" friction="%s" margin="%g" mass="%g"/>' % (
                               g.name, names[g.kind], ('mesh="%s_mesh"' % g.name) if g.kind == MESH else
                               'size="%s"' % ' '.join('%.9g' % v for v in g.size),
                               ' '.join('%.9g' % v for v in g.pos), ' '.join('%.9g' % v for v in g.quat),
                               g.contype, g.conaffinity, g.condim, ' '.join('%g' % v for v in g.friction),
                               g.margin, g.mass))
            for s in b.sites:
                out.append(ind + '<site name="%s" pos="%s"/>' % (s.name, ' '.join('%g' % v for v in s['pos'])))
        while len(stack) > 1:
            stack.pop()
            out.append('  ' * depth[stack[-1]] + '  </body>')
        out.append('  </worldbody>')
        out.append('  <actuator>')
        for a in self.actuators:
            out.append('    <general joint="%s" gaintype="%s" biastype="%s" gainprm="%s" biasprm="%s"%s%s/>' % (
                a['joint_name'], 'fixed' if a['gaintype'] == 0 else 'affine',
                'none' if a['biastype'] == 0 else 'affine', ' '.join('%g' % v for v in a['gainprm']),
                ' '.join('%g' % v for v in a['biasprm']),
                ' ctrllimited="true" ctrlrange="%g %g"' % tuple(a['ctrlrange']) if a.get('ctrlrange') else '',
                ' forcelimited="true" forcerange="%g %g"' % tuple(a['forcerange']) if a.get('forcerange') else ''))
        out.append('  </actuator>')
        out.append('</mujoco>')
        return '\n'.join(out)


class _Site(dict):
    @property
    def name(self):
        return self['name']


def parameter_rows(scenes):
    """Per-world parameter rows from compiled scenes of one topology.

    Returns {real array name: [len(scenes), length]} for every real array
    that differs between the scenes; with native.PackedModel(scenes[0],
    rows=...) world w then runs scenes[w % len(scenes)]'s arrays, derived ones
    included (inertias, AABBs, invweights).  The scenes must agree on sizes,
    int arrays, scalars and options, except meaninertia, which stays the first
    scene's (one value per model: the reference's Newton leaves take
    m.stat.meaninertia as one scalar, host/runtime/newton/mjwarp_linesearch.py:79)."""
    scenes = list(scenes)
    if not scenes:
        raise ValueError('parameter_rows needs at least one scene')
    first = scenes[0]
    for k, other in enumerate(scenes[1:], 1):
        if other.sizes != first.sizes:
            raise ValueError('scene %d has other sizes than scene 0' % k)
        for name, value in first.ints.items():
            if not np.array_equal(np.asarray(value), np.asarray(other.ints[name])):
                raise ValueError('scene %d differs from scene 0 in int array %s (topology)' % (k, name))
        for name, value in first.scalars.items():
            if name != 'meaninertia' and value != other.scalars[name]:
                raise ValueError('scene %d differs from scene 0 in scalar %s' % (k, name))
        for name in set(first.options) | set(other.options):
            if first.options.get(name) != other.options.get(name):
                raise ValueError('scene %d differs from scene 0 in scalar option %s' % (k, name))
    rows = {}
    for name in first.reals:
        stack = np.stack([np.asarray(sc.reals[name], np.float64).reshape(-1) for sc in scenes])
        if np.any(stack != stack[0]):
            rows[name] = stack
    return rows


def _panda(bodies, link_radius=0.06, box_margin=0.001):
    """Append a Franka-like arm (7 hinges + 2 finger slides) under the world;
    the finger pads are boxes with margin `box_margin`."""
    ARM, OBJ = 2, 1   # contype bits: arm geoms never collide with each other
    links = [  # (pos, quat, capsule half-length, capsule centre offset/axis quat)
        ((0, 0, 0.333), (1, 0, 0, 0)),
        ((0, 0, 0), axis_quat((1, 0, 0), -math.pi / 2)),
        ((0, -0.316, 0), axis_quat((1, 0, 0), math.pi / 2)),
        ((0.0825, 0, 0), axis_quat((1, 0, 0), math.pi / 2)),
        ((-0.0825, 0.384, 0), axis_quat((1, 0, 0), -math.pi / 2)),
        ((0, 0, 0), axis_quat((1, 0, 0), math.pi / 2)),
        ((0.088, 0, 0), axis_quat((1, 0, 0), math.pi / 2)),
    ]
    capsule = [  # per link: (centre, quat, half-length) in the link frame
        ((0, 0, -0.10), (1, 0, 0, 0), 0.06),
        ((0, -0.08, 0), axis_quat((1, 0, 0), math.pi / 2), 0.06),
        ((0, 0, -0.08), (1, 0, 0, 0), 0.07),
        ((-0.04, 0.09, 0), axis_quat((1, 0, 0), math.pi / 2), 0.08),
        ((0, 0, -0.14), (1, 0, 0, 0), 0.09),
        ((0.044, 0, 0), axis_quat((0, 1, 0), math.pi / 2), 0.03),
        ((0, 0, 0.05), (1, 0, 0, 0), 0.03),
    ]
    parent = 0
    joints = []
    for k, ((pos, quat), (cpos, cquat, hl)) in enumerate(zip(links, capsule)):
        b = Body('link%d' % (k + 1), parent, pos, tuple(quat))
        b.joints.append(Joint('joint%d' % (k + 1), HINGE, (0, 0, 1), range=PANDA_RANGES[k],
                              damping=0.1, armature=0.1, frictionloss=0.1))
        b.geoms.append(Geom('link%d_col' % (k + 1), CAPSULE, (link_radius, hl), cpos, tuple(cquat),
                            contype=ARM, conaffinity=OBJ, mass=PANDA_MASS[k]))
        bodies.append(b)
        parent = len(bodies) - 1
        joints.append(k)
    hand = Body('hand', parent, (0, 0, 0.107), tuple(axis_quat((0, 0, 1), -math.pi / 4)))
    hand.geoms.append(Geom('hand_col', CAPSULE, (0.03, 0.07), (0, 0, 0.02), tuple(axis_quat((1, 0, 0), math.pi / 2)),
                           contype=ARM, conaffinity=OBJ, mass=0.73))
    hand.sites.append(_Site(name='grip_site', pos=(0.0, 0.0, 0.1034)))
    bodies.append(hand)
    hand_id = len(bodies) - 1
    for side, (lo, hi) in ((1, (0.0, 0.04)), (-1, (-0.04, 0.0))):
        f = Body('finger%d' % (1 if side > 0 else 2), hand_id, (0, 0, 0.0584))
        f.joints.append(Joint('finger_joint%d' % (1 if side > 0 else 2), SLIDE, (0, 1, 0), range=(lo, hi),
                              damping=100.0, armature=1.0, frictionloss=1.0))
        f.geoms.append(Geom('finger%d_pad' % (1 if side > 0 else 2), BOX, (0.01, 0.01, 0.025),
                            (0, 0.012 * side, 0.028), contype=ARM, conaffinity=OBJ, margin=box_margin, mass=0.1))
        bodies.append(f)
    njoint = 9
    actuators = []
    for k in range(7):
        actuators.append(dict(joint=k, joint_name='joint%d' % (k + 1), gaintype=0, biastype=0,
                              gainprm=(1.0, 0, 0), biasprm=(0.0, 0, 0),
                              ctrlrange=(-PANDA_TORQUE[k], PANDA_TORQUE[k])))
    for k, rng in ((7, (0.0, 0.04)), (8, (-0.04, 0.0))):
        actuators.append(dict(joint=k, joint_name='finger_joint%d' % (k - 6), gaintype=0, biastype=1,
                              gainprm=(1000.0, 0, 0), biasprm=(0.0, -1000.0, 0), ctrlrange=rng,
                              forcerange=(-20.0, 20.0)))
    controller = dict(site='grip_site', joints=list(range(7)), gripper_joints=[7, 8],
                      actuators=list(range(9)), kp=150.0, damping_ratio=1.0,
                      q0=PANDA_INIT_QPOS, uncouple=True)
    assert njoint == 9
    return actuators, controller


def _ee_xy(scene):
    from . import kinematics_host as kh
    q = scene.reals['qpos0'].copy()
    for k, j in enumerate(scene.controller['joints']):
        q[scene.ints['jnt_qposadr'][j]] = scene.controller['q0'][k]
    st = kh.forward_position(scene, q)
    return st['site_xpos'][scene.sizes['ee_site']][:2]


def scene_a(seed=0, cone='elliptic', nconmax=32, njmax=None, iterations=50, ls_iterations=50,
            tolerance=1e-8, box_margin=0.001):
    """BASELINE scene A: arm + gripper + plane + 3 free boxes (nq=30, nv=27).

    The boxes and finger pads carry a margin of `box_margin`; with 0, box-box
    pairs take the convex path and its box manifold, as in a LIBERO scene whose
    boxes have no margin."""
    rng = np.random.default_rng([seed, 0xA])
    bodies = [Body('world', -1)]
    bodies[0].geoms.append(Geom('floor', PLANE, (0, 0, 0.05), contype=1, conaffinity=3))
    actuators, controller = _panda(bodies, box_margin=box_margin)
    objects = []
    for k in range(3):
        half = rng.uniform(0.02, 0.05, 3)
        mass = rng.uniform(0.05, 0.3)
        b = Body('box%d' % k, 0, (0.5, 0.0, half[2]))
        b.joints.append(Joint('box%d_free' % k, FREE))
        b.geoms.append(Geom('box%d_geom' % k, BOX, tuple(half), contype=1, conaffinity=3,
                            friction=(1.0, 0.005, 0.0001), margin=box_margin, mass=mass))
        bodies.append(b)
        objects.append(dict(id=len(bodies) - 1, radius=float(np.linalg.norm(half[:2])), rbound=float(np.linalg.norm(half)),
                            rest_z=float(half[2]),
                            drop=None))
    opt = dict(timestep=0.002, iterations=iterations, ls_iterations=ls_iterations, tolerance=tolerance,
               cone=1 if cone == 'elliptic' else 0, impratio=1.0, ls_tolerance=0.01)
    scene = Scene('scene_a', bodies, actuators, opt, dict(nconmax=nconmax, njmax=njmax), controller)
    scene.objects = objects
    scene.object_square = 0.4
    scene.object_center = _ee_xy(scene)
    scene.substeps = 25
    return scene


def scene_b(seed=0, cone='elliptic', nconmax=96, njmax=None, iterations=50, ls_iterations=50,
            tolerance=1e-8, hull_points=32, epa_iterations=32, ccd_tolerance=1e-6, box_margin=0.001):
    """BASELINE scene B: scene A's arm plus 12 dropped free objects (nq=93, nv=81).

    4 boxes (half-extents U[0.02,0.05]), 4 capsules (radius U[0.015,0.04],
    half-length U[0.02,0.05]), 2 spheres (radius U[0.02,0.05]) and 2 convex
    hulls of 32 random points on an ellipsoid with semi-axes U[0.02,0.06];
    masses U[0.05,0.3] kg, friction 1; dropped from z U[0.05,0.15] m with a
    random orientation.  Boxes (finger pads included) carry a margin of
    `box_margin`, hulls a 1 mm margin."""
    rng = np.random.default_rng([seed, 0xB])
    bodies = [Body('world', -1)]
    bodies[0].geoms.append(Geom('floor', PLANE, (0, 0, 0.05), contype=1, conaffinity=3))
    actuators, controller = _panda(bodies, box_margin=box_margin)
    objects = []
    kinds = [BOX] * 4 + [CAPSULE] * 4 + [SPHERE] * 2 + [MESH] * 2
    for k, kind in enumerate(kinds):
        mass = rng.uniform(0.05, 0.3)
        mesh, margin = None, 0.0
        if kind == BOX:
            size = tuple(rng.uniform(0.02, 0.05, 3))
            radius, margin = float(np.linalg.norm(size)), box_margin
        elif kind == CAPSULE:
            size = (rng.uniform(0.015, 0.04), rng.uniform(0.02, 0.05))
            radius = size[0] + size[1]
        elif kind == SPHERE:
            size = (rng.uniform(0.02, 0.05),)
            radius = size[0]
        else:
            axes = rng.uniform(0.02, 0.06, 3)
            d = rng.normal(size=(hull_points, 3))
            d /= np.linalg.norm(d, axis=1, keepdims=True)
            mesh = convex_mesh(d * axes)
            size, margin = tuple(np.ptp(mesh['vert'], axis=0) / 2), 0.001
            radius = float(np.max(np.linalg.norm(mesh['vert'], axis=1)))
        name = {BOX: 'box', CAPSULE: 'capsule', SPHERE: 'sphere', MESH: 'hull'}[kind]
        b = Body('%s%d' % (name, k), 0, (0.5, 0.0, 0.1))
        b.joints.append(Joint('%s%d_free' % (name, k), FREE))
        b.geoms.append(Geom('%s%d_geom' % (name, k), kind, size, contype=1, conaffinity=3,
                            friction=(1.0, 0.005, 0.0001), margin=margin, mass=mass, mesh=mesh))
        bodies.append(b)
        objects.append(dict(id=len(bodies) - 1, radius=radius, rest_z=None, drop=(0.05, 0.15), tumble=True))
    opt = dict(timestep=0.002, iterations=iterations, ls_iterations=ls_iterations, tolerance=tolerance,
               cone=1 if cone == 'elliptic' else 0, impratio=1.0, ls_tolerance=0.01, epa_iterations=epa_iterations,
               ccd_tolerance=ccd_tolerance)
    scene = Scene('scene_b', bodies, actuators, opt, dict(nconmax=nconmax, njmax=njmax), controller)
    scene.objects = objects
    scene.object_square = 0.5
    scene.object_center = _ee_xy(scene)
    scene.substeps = 25
    return scene
