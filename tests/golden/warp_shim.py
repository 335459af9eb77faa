"""A CPU stand-in for the subset of NVIDIA Warp used by dsl_splat's gs3d and
RaDe-GS kernels.

Test infrastructure only.  warp-lang is not installable here, so to pin the
CPU oracle against the reference itself, make_golden.py imports the
reference's modules with this object registered as `warp` and executes the
reference's own kernel source on the CPU:

* `@wp.func` / `@wp.kernel` bodies are re-compiled from their source with
  every float literal and `float(...)` cast typed float32 (numpy scalars),
  as Warp types them; integer arithmetic stays Python ints;
* vectors, matrices and arrays are small float32 containers with Warp's
  component-wise semantics;
* `@wp.func_native` snippets with arithmetic (fmaf, the GLM rotation,
  __float_as_uint) are compiled from the reference's snippet text with g++
  (-ffp-contract=off) and called through ctypes; the block primitives
  (__syncthreads, __syncthreads_count, __shared__ arrays) are emulated by
  running each 256-thread block as 256 Python threads with a barrier;
  the warp intrinsics (__any_sync, and the shuffle-down lane sums of
  primitives/warp.py) exchange values among the 32 threads of a warp and
  reproduce the shuffle-down tree's float32 summation order;
* `wp.exp` is the same Cody-Waite exp the oracle and the CUDA kernels use
  (a deliberate substitution; CUDA's expf is not reproducible here), the
  AAA snippets' atan2f / tanf / logf are the oracle's own (see
  _SUBSTITUTIONS), and
  `norm3df` (rade/projection.py:33) is sqrtf(x*x + y*y + z*z) in IEEE
  float32, as the oracle and the CUDA kernels compute the sort distance.

Arithmetic is IEEE float32 without contraction, i.e. the reference's kernel
logic, not Warp's NVRTC code generation.
"""

from __future__ import annotations

import ast
import ctypes
import inspect
import os
import subprocess
import sys
import tempfile
import textwrap
import threading
import types

import numpy as np

F32 = np.float32
F64 = np.float64

_state = threading.local()
_atomic_lock = threading.Lock()


def _f64_mode() -> bool:
    return getattr(_state, "f64", False)


def _wp_f32(x):
    """float(...) and float literals inside kernels."""
    if isinstance(x, Vec):
        raise TypeError("float() of a vector")
    return F64(x) if _f64_mode() else F32(x)


def _wp_int(x):
    if isinstance(x, (np.floating, float)):
        if np.isnan(x):
            return 0
        return int(np.trunc(x))
    return int(x)


def _cast(x, dtype):
    if dtype is float or dtype is F32:
        return _wp_f32(x)
    if dtype is int or dtype is np.int32:
        return _wp_int(x)
    if dtype is bool:
        return bool(x)
    return dtype(x)


# ---- value types -------------------------------------------------------------

class Vec:
    length = 0
    dtype = float
    __slots__ = ("v",)
    __array_ufunc__ = None  # numpy scalars defer to Vec's operators

    def __init__(self, *args):
        n = type(self).length
        if len(args) == 0:
            self.v = [_cast(0, self.dtype) for _ in range(n)]
        elif len(args) == 1 and isinstance(args[0], Vec):
            self.v = [_cast(a, self.dtype) for a in args[0].v]
        elif len(args) == 1:
            self.v = [_cast(args[0], self.dtype) for _ in range(n)]
        else:
            assert len(args) == n, (type(self).__name__, len(args))
            self.v = [_cast(a, self.dtype) for a in args]

    def __getitem__(self, i):
        return self.v[i]

    def __setitem__(self, i, value):
        self.v[i] = _cast(value, self.dtype)

    def __len__(self):
        return len(self.v)

    def _new(self, values):
        out = type(self).__new__(type(self))
        out.v = [_cast(a, self.dtype) for a in values]
        return out

    def __add__(self, o):
        return self._new([a + b for a, b in zip(self.v, o.v)])

    def __sub__(self, o):
        return self._new([a - b for a, b in zip(self.v, o.v)])

    def __mul__(self, s):
        if isinstance(s, Vec):
            raise TypeError("vector * vector")
        return self._new([a * s for a in self.v])

    def __rmul__(self, s):
        return self._new([s * a for a in self.v])

    def __truediv__(self, s):
        return self._new([a / s for a in self.v])

    def __neg__(self):
        return self._new([-a for a in self.v])

    def __repr__(self):
        return f"{type(self).__name__}({', '.join(str(a) for a in self.v)})"


_vec_types: dict = {}


def vector(length, dtype=float):
    key = (length, dtype)
    if key not in _vec_types:
        _vec_types[key] = type(f"vec{length}", (Vec,), {"length": length, "dtype": dtype,
                                                         "__slots__": ()})
    return _vec_types[key]


class Mat:
    rows = cols = 0
    __slots__ = ("m",)
    __array_ufunc__ = None

    def __init__(self, *args):
        R, C = type(self).rows, type(self).cols
        if len(args) == 0:
            self.m = [[_wp_f32(0) for _ in range(C)] for _ in range(R)]
        elif len(args) == 1 and isinstance(args[0], Mat):
            self.m = [list(r) for r in args[0].m]
        elif len(args) == 1:  # Warp fills every entry with the scalar
            self.m = [[_wp_f32(args[0]) for _ in range(C)] for _ in range(R)]
        else:
            assert len(args) == R * C
            self.m = [[_wp_f32(args[r * C + c]) for c in range(C)] for r in range(R)]

    def __getitem__(self, idx):
        if isinstance(idx, tuple):
            return self.m[idx[0]][idx[1]]
        return vector(type(self).cols)(*self.m[idx])

    def __setitem__(self, idx, value):
        if isinstance(idx, tuple):
            self.m[idx[0]][idx[1]] = _wp_f32(value)
        else:  # a whole row from a vector
            self.m[idx] = [_wp_f32(a) for a in value.v]

    def __mul__(self, o):
        """Matrix-vector or matrix-matrix product, each sum left to right."""
        if isinstance(o, Mat):
            out = matrix(type(self).rows, type(o).cols)()
            for r, row in enumerate(self.m):
                for c in range(type(o).cols):
                    acc = row[0] * o.m[0][c]
                    for k in range(1, len(row)):
                        acc = acc + row[k] * o.m[k][c]
                    out.m[r][c] = acc
            return out
        if not isinstance(o, Vec):  # matrix * scalar, element-wise
            out = type(self)()
            out.m = [[_wp_f32(a * o) for a in row] for row in self.m]
            return out
        out = []
        for row in self.m:
            acc = row[0] * o.v[0]
            for a, b in zip(row[1:], o.v[1:]):
                acc = acc + a * b
            out.append(acc)
        return vector(type(self).rows)(*out)


_mat_types: dict = {}


def matrix(rows, cols):
    key = (rows, cols)
    if key not in _mat_types:
        _mat_types[key] = type(f"mat{rows}{cols}", (Mat,), {"rows": rows, "cols": cols,
                                                             "__slots__": ()})
    return _mat_types[key]


class Array:
    """Kernel view of a numpy array; vector dtypes read/write whole rows."""

    def __init__(self, data: np.ndarray, dtype=None):
        self.data = data
        self.dtype = dtype
        self.shape = data.shape if dtype is None or not isinstance(dtype, type) or not (
            issubclass(dtype, (Vec, Mat))) else data.shape[:1]

    def _is_vec(self):
        return isinstance(self.dtype, type) and issubclass(self.dtype, Vec)

    def _is_mat(self):
        return isinstance(self.dtype, type) and issubclass(self.dtype, Mat)

    def __getitem__(self, idx):
        if self._is_vec():
            return self.dtype(*self.data[idx])
        if self._is_mat():
            return self.dtype(*self.data[idx].ravel())
        v = self.data[idx]
        if self.data.dtype == np.float32:
            return _wp_f32(v)
        if self.data.dtype == np.bool_:
            return bool(v)
        if self.data.dtype == np.uint64:
            return np.uint64(v)
        return int(v)

    def __setitem__(self, idx, value):
        if self._is_vec():
            self.data[idx] = [float(a) for a in value.v]
        elif self._is_mat():
            self.data[idx] = [[float(a) for a in row] for row in value.m]
        else:
            self.data[idx] = value


class _ArrayType:
    """What `wp.array(dtype=...)` evaluates to inside annotations."""

    def __init__(self, dtype=None, ndim=1, **kw):
        self.dtype, self.ndim = dtype, ndim


# ---- kernel / func compilation --------------------------------------------------

class _TypeLiterals(ast.NodeTransformer):
    def visit_Constant(self, node):
        if isinstance(node.value, float):
            return ast.copy_location(
                ast.Call(func=ast.Name("__wp_f32", ast.Load()), args=[node], keywords=[]), node)
        return node

    def visit_Call(self, node):
        self.generic_visit(node)
        if isinstance(node.func, ast.Name) and node.func.id == "float":
            node.func = ast.Name("__wp_f32", ast.Load())
        elif isinstance(node.func, ast.Name) and node.func.id == "int":
            node.func = ast.Name("__wp_int", ast.Load())
        return node


def _recompile(fn):
    """fn's source with Warp literal typing, closed over fn's current free variables."""
    src = textwrap.dedent(inspect.getsource(fn))
    tree = ast.parse(src)
    fdef = tree.body[0]
    fdef.decorator_list = []
    fdef = _TypeLiterals().visit(fdef)
    free = fn.__code__.co_freevars
    outer = ast.FunctionDef(
        name="__wp_outer",
        args=ast.arguments(posonlyargs=[], args=[ast.arg(arg=v) for v in free], vararg=None,
                           kwonlyargs=[], kw_defaults=[], kwarg=None, defaults=[]),
        body=[fdef, ast.Return(ast.Name(fdef.name, ast.Load()))], decorator_list=[],
        returns=None, type_params=[])
    module = ast.Module(body=[outer], type_ignores=[])
    ast.fix_missing_locations(module)
    g = fn.__globals__
    g.setdefault("__wp_f32", _wp_f32)
    g.setdefault("__wp_int", _wp_int)
    ns: dict = {}
    exec(compile(module, inspect.getsourcefile(fn) or "<kernel>", "exec"), g, ns)
    cells = [c.cell_contents for c in (fn.__closure__ or ())]
    return ns["__wp_outer"](*cells)


class Kernel:
    def __init__(self, fn, options):
        self.fn = _recompile(fn)
        self.key = fn.__name__
        self.options = options

    def __call__(self, *args):
        return self.fn(*args)


def kernel(fn=None, **options):
    if fn is None:
        return lambda f: Kernel(f, options)
    return Kernel(fn, options)


def func(fn):
    if fn.__name__ in _FUNC_NATIVES and fn.__module__.endswith("primitives.warp"):
        return _FUNC_NATIVES[fn.__name__]
    out = _recompile(fn)
    out.__wp_source__ = fn
    return out


def func_grad(target):
    def deco(fn):
        return fn  # custom adjoints are not executed by the stand-in
    return deco


class _Adjoint(dict):
    pass


adjoint = _Adjoint()


# ---- native snippets -----------------------------------------------------------------

_NATIVE_HEADER = r"""
#include <cmath>
#include <cstdint>
#include <cstring>
#include <type_traits>
namespace wp {
template <int N, typename T> struct vec_t {
  T c[N];
  vec_t() { for (int i = 0; i < N; ++i) c[i] = T(0); }
  explicit vec_t(T s) { for (int i = 0; i < N; ++i) c[i] = s; }  // Warp fills
  template <typename... A, typename = std::enable_if_t<(sizeof...(A) >= 2)>>
  vec_t(A... a) : c{static_cast<T>(a)...} {}
  T& operator[](int i) { return c[i]; }
  const T& operator[](int i) const { return c[i]; }
};
template <int N, typename T> vec_t<N, T> operator+(vec_t<N, T> a, const vec_t<N, T>& b) {
  for (int i = 0; i < N; ++i) a[i] = a[i] + b[i];
  return a;
}
template <int N, typename T> vec_t<N, T> operator-(vec_t<N, T> a, const vec_t<N, T>& b) {
  for (int i = 0; i < N; ++i) a[i] = a[i] - b[i];
  return a;
}
template <int N, typename T> vec_t<N, T> operator*(vec_t<N, T> a, T s) {
  for (int i = 0; i < N; ++i) a[i] = a[i] * s;
  return a;
}
template <int N, typename T> vec_t<N, T> operator*(T s, vec_t<N, T> a) {
  for (int i = 0; i < N; ++i) a[i] = s * a[i];
  return a;
}
template <int N, typename T> vec_t<N, T> cw_mul(vec_t<N, T> a, const vec_t<N, T>& b) {
  for (int i = 0; i < N; ++i) a[i] = a[i] * b[i];
  return a;
}
template <int R, int C, typename T> struct mat_t {
  T data[R][C];
  mat_t() { for (int i = 0; i < R * C; ++i) data[i / C][i % C] = T(0); }
  explicit mat_t(T s) { for (int i = 0; i < R * C; ++i) data[i / C][i % C] = s; }
  template <typename... A, typename = std::enable_if_t<(sizeof...(A) >= 2)>>
  mat_t(A... a) {
    const T v[] = {static_cast<T>(a)...};
    for (int i = 0; i < R * C; ++i) data[i / C][i % C] = v[i];
  }
  vec_t<C, T> get_row(int r) const {
    vec_t<C, T> out;
    for (int i = 0; i < C; ++i) out[i] = data[r][i];
    return out;
  }
};
}
static inline float __fmul_rn(float a, float b) { return a * b; }
static inline float __fadd_rn(float a, float b) { return a + b; }
static inline float __fsub_rn(float a, float b) { return a - b; }
static inline float __frcp_rn(float a) { return 1.0f / a; }  // correctly rounded
static inline uint32_t __float_as_uint(float v) { uint32_t u; std::memcpy(&u, &v, 4); return u; }
static inline float norm3df(float a, float b, float c) { return std::sqrt(a * a + b * b + c * c); }
"""

# Warp-cooperative snippets (ballot / shuffle across the 32 lanes of a warp)
# run as 32 std::threads per warp; every intrinsic is an exchange through
# one slot per lane between two barriers, so all lanes must reach it, as on
# the GPU.  Arrays are wp::array_t views with .data and .shape[0].
WARP_LANES_HEADER = r"""
#include <algorithm>
#include <barrier>
#include <thread>
#include <vector>
using std::max;
using std::min;
namespace wp {
template <typename T> struct array_t {
  T* data;
  int shape[1];
};
}
struct Dim3 { int x; };
struct WarpLanes {
  std::barrier<> bar{32};
  uint64_t slot[32];
};
thread_local Dim3 threadIdx;
thread_local WarpLanes* warp_lanes;
static inline unsigned __ballot_sync(unsigned, bool predicate) {
  warp_lanes->slot[threadIdx.x & 31] = predicate ? 1u : 0u;
  warp_lanes->bar.arrive_and_wait();
  unsigned out = 0;
  for (int l = 0; l < 32; ++l) out |= static_cast<unsigned>(warp_lanes->slot[l]) << l;
  warp_lanes->bar.arrive_and_wait();
  return out;
}
template <typename T> static inline T __shfl_sync(unsigned, T value, int source) {
  static_assert(sizeof(T) <= 8, "shuffle of a scalar");
  uint64_t bits = 0;
  std::memcpy(&bits, &value, sizeof(T));
  warp_lanes->slot[threadIdx.x & 31] = bits;
  warp_lanes->bar.arrive_and_wait();
  bits = warp_lanes->slot[source & 31];
  warp_lanes->bar.arrive_and_wait();
  T out;
  std::memcpy(&out, &bits, sizeof(T));
  return out;
}
static inline int __popc(unsigned x) { return __builtin_popcount(x); }
static inline int __ffs(int x) { return __builtin_ffs(x); }
// run body(thread index) over `threads` lanes (a multiple of 32), one warp
// of real threads at a time
template <typename F> static void run_warps(int threads, F body) {
  for (int start = 0; start < threads; start += 32) {
    WarpLanes lanes;
    std::vector<std::thread> pool;
    for (int lane = 0; lane < 32; ++lane)
      pool.emplace_back([&, lane] {
        threadIdx.x = lane;
        warp_lanes = &lanes;
        body(start + lane);
      });
    for (auto& t : pool) t.join();
  }
}
"""


# The transcendental functions on the AAA decision path (aaa/native_geometry.py's
# atan2f / tanf, aaa/binning_native.py's logf) are the oracle's own
# implementations in every snippet (oracle/aaa_oracle.cpp, splat_oracle.cpp),
# the ones the CUDA kernels use too: the host libm's float versions are not
# correctly rounded, and the tile bounds they feed are integers.  Defined
# after every library header, so only snippet text is affected.
_ORACLE_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(
    os.path.abspath(__file__)))), "oracle")
_SUBSTITUTIONS = r"""
extern "C" float oracle_atan2f(float, float);
extern "C" float oracle_tanf(float);
extern "C" float oracle_logf(float);
#define atan2f oracle_atan2f
#define tanf oracle_tanf
#define logf oracle_logf
"""
_LINK_ORACLE = ["-L" + _ORACLE_DIR, "-l:libsplat_oracle.so", "-Wl,-rpath," + _ORACLE_DIR]


def compile_warp_snippet(source: str, name: str):
    """g++ a C++ translation unit made of the float32 prelude, the warp-lane
    prelude and `source`; returns the ctypes library."""
    tmp = tempfile.mkdtemp(prefix="warp_shim_")
    path = os.path.join(tmp, f"{name}.cpp")
    with open(path, "w") as f:
        f.write(_NATIVE_HEADER + WARP_LANES_HEADER + _SUBSTITUTIONS + source)
    so = os.path.join(tmp, f"{name}.so")
    subprocess.run(["g++", "-O1", "-std=c++20", "-pthread", "-fPIC", "-shared",
                    "-ffp-contract=off", "-march=x86-64-v3", "-Wno-unknown-pragmas", "-o", so,
                    path, *_LINK_ORACLE], check=True)
    lib = ctypes.CDLL(so)
    _native_libs[name] = lib
    return lib


_C_TYPES = {}  # annotation -> (c type, n floats, kind)


def _c_type(ann):
    if ann is float or ann is F32:
        return "float", 1, "scalar"
    if ann is np.uint32 or ann is uint32:
        return "uint32_t", 1, "u32"
    if ann is bool:
        return "bool", 1, "bool"
    if ann is int:
        return "int", 1, "int"
    if isinstance(ann, type) and issubclass(ann, Vec):
        return f"wp::vec_t<{ann.length},float>", ann.length, "vec"
    if isinstance(ann, type) and issubclass(ann, Mat):
        return f"wp::mat_t<{ann.rows},{ann.cols},float>", ann.rows * ann.cols, "mat"
    raise TypeError(f"unsupported native annotation {ann!r}")


_native_libs: dict = {}
_BLOCK_NATIVES = {}
# natives of one reference module (name clashes across modules: the AAA
# renderer's shared_ids / any_active differ from gs3d's)
_MODULE_NATIVES = {}


def _compile_native(name, snippet, params, ret):
    """Compile one reference snippet into extern "C" float-array entry points."""
    args, unpack = [], []
    for i, (pname, ann) in enumerate(params):
        ctype, n, kind = _c_type(ann)
        args.append(f"const float* a{i}")
        if kind == "scalar":
            unpack.append(f"const float {pname} = a{i}[0];")
        elif kind == "vec":
            unpack.append(f"{ctype} {pname}; for (int k = 0; k < {n}; ++k) {pname}[k] = a{i}[k];")
        elif kind == "mat":
            cols = ann.cols
            unpack.append(f"{ctype} {pname}; for (int k = 0; k < {n}; ++k) "
                          f"{pname}.data[k / {cols}][k % {cols}] = a{i}[k];")
        elif kind == "bool":
            unpack.append(f"const bool {pname} = a{i}[0] != 0.0f;")
        elif kind == "int":
            unpack.append(f"const int {pname} = static_cast<int>(a{i}[0]);")
        else:
            raise TypeError(kind)
    rtype, rn, rkind = _c_type(ret)
    body = textwrap.indent(snippet.strip(), "  ")
    sig = ", ".join(f"{_c_type(ann)[0]} {pname}" for pname, ann in params)
    src = _NATIVE_HEADER + _SUBSTITUTIONS + f"\nstatic {rtype} impl_{name}({sig}) {{\n{body}\n}}\n"
    call = ", ".join(pname for pname, _ in params)
    cols = getattr(ret, "cols", 1)
    store = {"scalar": "out[0] = r;",
             "u32": "std::memcpy(out, &r, 4);",
             "vec": f"for (int k = 0; k < {rn}; ++k) out[k] = r[k];",
             "mat": f"for (int k = 0; k < {rn}; ++k) out[k] = r.data[k / {cols}][k % {cols}];"}[rkind]
    src += (f'extern "C" void call_{name}({", ".join(args)}, float* out) {{\n'
            + "\n".join("  " + u for u in unpack)
            + f"\n  const {rtype} r = impl_{name}({call});\n  {store}\n}}\n")
    tmp = tempfile.mkdtemp(prefix="warp_shim_")
    path = os.path.join(tmp, f"{name}.cpp")
    with open(path, "w") as f:
        f.write(src)
    so = os.path.join(tmp, f"{name}.so")
    subprocess.run(["g++", "-O1", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off",
                    "-march=x86-64-v3", "-o", so, path, *_LINK_ORACLE], check=True)
    lib = ctypes.CDLL(so)
    fn = getattr(lib, f"call_{name}")
    fn.restype = None
    _native_libs[name] = lib
    return fn, rkind, rn, ret


def func_native(snippet, adj_snippet=None):
    def deco(fn):
        name = fn.__name__
        qualified = (fn.__module__, name)
        if qualified in _MODULE_NATIVES:
            return _MODULE_NATIVES[qualified]
        if name in _BLOCK_NATIVES:
            return _BLOCK_NATIVES[name]
        hints = {k: v for k, v in fn.__annotations__.items()}
        ret = hints.pop("return", None)  # None: a void snippet, not callable here
        params = list(hints.items())
        compiled = {}

        def call(*values):
            if "fn" not in compiled:
                compiled["fn"] = _compile_native(name, snippet, params, ret)
            cfn, rkind, rn, rtype = compiled["fn"]
            bufs = []
            for v, (_, ann) in zip(values, params):
                arr = (ctypes.c_float * max(1, _c_type(ann)[1]))()
                if isinstance(v, Vec):
                    for k, a in enumerate(v.v):
                        arr[k] = float(a)
                elif isinstance(v, Mat):
                    for k, a in enumerate(x for row in v.m for x in row):
                        arr[k] = float(a)
                else:
                    arr[0] = float(v)
                bufs.append(arr)
            out = (ctypes.c_float * rn)()
            cfn(*bufs, out)
            if rkind == "scalar":
                return F32(out[0])
            if rkind == "u32":
                return np.frombuffer(bytes(out), dtype=np.uint32)[0]
            if rkind == "vec":
                return rtype(*[F32(x) for x in out])
            return rtype(*[F32(x) for x in out])

        call.__name__ = name
        call.__wp_snippet__ = snippet
        return call
    return deco


# ---- block execution (barriers, shared memory) ----------------------------------------

class _Block:
    def __init__(self, size):
        self.size = size
        self.barrier = threading.Barrier(size)
        self.shared: dict = {}
        self.flags = [False] * size
        self.lock = threading.Lock()
        warps = (size + 31) // 32
        self.warp_barriers = [threading.Barrier(min(32, size - 32 * w)) for w in range(warps)]
        self.warp_slots = [[None] * 32 for _ in range(warps)]
        self.group_barriers: dict = {}

    def group_barrier(self, warp: int, mask: int):
        """The barrier of the lanes of `mask` in `warp` (__syncwarp(mask))."""
        key = (warp, mask)
        with self.lock:
            if key not in self.group_barriers:
                self.group_barriers[key] = threading.Barrier(bin(mask).count("1"))
            return self.group_barriers[key]

    def abort(self):
        self.barrier.abort()
        for b in self.warp_barriers:
            b.abort()
        with self.lock:
            for b in self.group_barriers.values():
                b.abort()


def _block() -> _Block:
    return _state.block


def _synchronize():
    _block().barrier.wait()


def _all_done(done):
    b = _block()
    b.flags[_state.lane] = bool(done)
    b.barrier.wait()
    count = sum(b.flags)
    b.barrier.wait()
    return count == b.size


def _warp_exchange(value):
    """Every lane's value, in lane order, for the 32 threads of this warp."""
    b = _block()
    w, lane = _state.lane // 32, _state.lane % 32
    b.warp_slots[w][lane] = value
    b.warp_barriers[w].wait()
    values = list(b.warp_slots[w])
    b.warp_barriers[w].wait()
    return values


def _any_active(predicate):
    """__any_sync(0xffffffff, predicate) (primitives/warp.py:12-13)."""
    return any(bool(v) for v in _warp_exchange(bool(predicate)))


def _shuffle_tree(values):
    """The float32 result of primitives/warp.py:20-25 in every lane: five
    __shfl_down_sync steps (16, 8, 4, 2, 1); a lane whose source is past the
    warp reads its own value, as __shfl_down_sync does."""
    v = list(values)
    n = len(v)
    for offset in (16, 8, 4, 2, 1):
        v = [v[i] + (v[i + offset] if i + offset < n else v[i]) for i in range(n)]
    return v


def _sum_lanes(value):
    return _shuffle_tree(_warp_exchange(value))[_state.lane % 32]


def _sum_vector_lanes(value):
    """primitives/warp.py:28-32: each component reduced with sum_lanes."""
    rows = _warp_exchange(value)
    lane = _state.lane % 32
    out = [_shuffle_tree([r.v[k] for r in rows])[lane] for k in range(len(value.v))]
    return value._new(out)


def _shared_flat(kind, size):
    def make():
        b = _block()
        with b.lock:
            if kind not in b.shared:
                b.shared[kind] = Array(np.zeros(size, np.float32))
            return b.shared[kind]
    return make


def _shared_flat_int(kind, size):
    def make():
        b = _block()
        with b.lock:
            if kind not in b.shared:
                b.shared[kind] = Array(np.zeros(size, np.int32))
            return b.shared[kind]
    return make


def _shared(kind, dtype):
    def make():
        b = _block()
        with b.lock:
            if kind not in b.shared:
                if dtype is int:
                    b.shared[kind] = Array(np.zeros(b.size, np.int32))
                else:
                    b.shared[kind] = Array(np.zeros((b.size, dtype.length), np.float32), dtype)
            return b.shared[kind]
    return make


def _shared_rows(kind, rows, dtype):
    def make():
        b = _block()
        with b.lock:
            if kind not in b.shared:
                b.shared[kind] = Array(np.zeros((rows, dtype.length), np.float32), dtype)
            return b.shared[kind]
    return make


# ---- masked warp intrinsics of the AAA HIER renderer ----------------------------------
# aaa/render_warp_intrinsics.py: __syncwarp(mask), __any_sync, __popc(__ballot_sync)
# and __shfl_sync(mask, v, src, width) among the lanes of `mask` (all of which
# reach the call, as the renderer guarantees), through the warp's slots.

def _group_exchange(mask, value):
    b = _block()
    w, lane = _state.lane // 32, _state.lane % 32
    bar = b.group_barrier(w, int(mask))
    b.warp_slots[w][lane] = value
    bar.wait()
    values = list(b.warp_slots[w])
    bar.wait()
    return values


def _masked_sync(mask):
    b = _block()
    b.group_barrier(_state.lane // 32, int(mask)).wait()


def _masked_any(mask, predicate):
    m = int(mask)
    values = _group_exchange(m, bool(predicate))
    return any(values[l] for l in range(32) if (m >> l) & 1)


def _masked_count(mask, predicate):
    m = int(mask)
    values = _group_exchange(m, bool(predicate))
    return sum(1 for l in range(32) if (m >> l) & 1 and values[l])


def _masked_shuffle(mask, value, source, width):
    values = _group_exchange(int(mask), value)
    lane = _state.lane % 32
    return values[(lane & ~(int(width) - 1)) + int(source) % int(width)]


def _load_matrix(matrices, index):
    return matrices[int(index)]


def _reciprocal(value):
    return F32(1.0) / F32(value)  # __frcp_rn: the correctly rounded 1/x


def _global_atomic_add(values, index, value):
    with _atomic_lock:
        previous = F32(values.data[int(index)])
        values.data[int(index)] = previous + F32(value)
    return previous


# @wp.func bodies replaced by an equivalent of the same float32 arithmetic
# (lane exchange instead of five shuffles each)
_FUNC_NATIVES = {"sum_lanes": _sum_lanes, "sum_vector_lanes": _sum_vector_lanes}


def _install_block_natives():
    _BLOCK_NATIVES["synchronize"] = _synchronize
    _BLOCK_NATIVES["all_done"] = _all_done
    _BLOCK_NATIVES["shared_ids"] = _shared("ids", int)
    _BLOCK_NATIVES["shared_centers"] = _shared("centers", vector(2))
    _BLOCK_NATIVES["shared_conics"] = _shared("conics", vector(4))
    # rade/render.py:60-96: channel-major feature cache (up to 32 channels)
    # and the 512 staged (plane, normal) rows
    _BLOCK_NATIVES["shared_features"] = _shared_flat("features", 256 * 32)
    _BLOCK_NATIVES["shared_geometry"] = _shared_rows("geometry", 512, vector(3))
    _BLOCK_NATIVES["any_active"] = _any_active
    hier = "dsl_splat.aaa.render_warp_intrinsics"
    _MODULE_NATIVES[(hier, "shared_depths")] = _shared_flat("hier_depths", 1536)
    _MODULE_NATIVES[(hier, "shared_ids")] = _shared_flat_int("hier_ids", 1536)
    _MODULE_NATIVES[(hier, "sync")] = _masked_sync
    _MODULE_NATIVES[(hier, "any_active")] = _masked_any
    _MODULE_NATIVES[(hier, "count_active")] = _masked_count
    _MODULE_NATIVES[(hier, "shuffle_int")] = _masked_shuffle
    _MODULE_NATIVES[(hier, "shuffle_float")] = _masked_shuffle
    _MODULE_NATIVES[(hier, "load_matrix")] = _load_matrix
    _MODULE_NATIVES[("dsl_splat.aaa.render_warp_geometry", "reciprocal")] = _reciprocal
    _MODULE_NATIVES[("dsl_splat.primitives.atomics", "global_atomic_add")] = _global_atomic_add


def tid():
    return _state.tid


def tile(value):
    """wp.tile of one value per lane: the lane's own value."""
    return value


def tile_sum(value):
    """wp.tile_sum over a 32-lane tile: the lanes' values summed in lane
    order (exact for the integer counts it reduces here), as a 1-tile."""
    values = _warp_exchange(value)
    total = values[0]
    for v in values[1:]:
        total = total + v
    return [total]


def launch_tiled(kernel_obj: Kernel, dim: int, args, block_dim: int = 32):
    """wp.launch_tiled: dim blocks of block_dim real threads, wp.tid() =
    (block, lane)."""
    errors = []

    def worker(blk, index, lane):
        _state.block, _state.tid, _state.lane = blk, (index, lane), lane
        try:
            kernel_obj(*args)
        except BaseException as e:  # surface thread failures
            errors.append(e)
            blk.abort()

    for index in range(dim):
        blk = _Block(block_dim)
        threads = [threading.Thread(target=worker, args=(blk, index, lane))
                   for lane in range(block_dim)]
        for th in threads:
            th.start()
        for th in threads:
            th.join()
        if errors:
            raise errors[0]


def launch(kernel_obj: Kernel, dim: int, args, block: int | None = None):
    """Run a kernel over dim threads; block-cooperative kernels as real blocks."""
    if block is None:
        for t in range(dim):
            _state.tid = t
            kernel_obj(*args)
        return
    errors = []

    def worker(blk, t, lane):
        _state.block, _state.tid, _state.lane = blk, t, lane
        try:
            kernel_obj(*args)
        except BaseException as e:  # surface thread failures
            errors.append(e)
            blk.abort()

    for start in range(0, dim, block):
        blk = _Block(block)
        threads = [threading.Thread(target=worker, args=(blk, start + lane, lane))
                   for lane in range(block)]
        for th in threads:
            th.start()
        for th in threads:
            th.join()
        if errors:
            raise errors[0]


# ---- builtins ------------------------------------------------------------------------

def _elementwise(f, a, b):
    if isinstance(a, Vec):
        return a._new([f(x, y) for x, y in zip(a.v, b.v)])
    return f(a, b)


def min(a, b):  # noqa: A001
    return _elementwise(lambda x, y: x if x < y else y, a, b)


def max(a, b):  # noqa: A001
    return _elementwise(lambda x, y: x if x > y else y, a, b)


def clamp(x, a, b):
    return min(max(a, x), b)


def sqrt(x):
    return type(x)(np.sqrt(x)) if isinstance(x, np.floating) else np.sqrt(F32(x))


def ceil(x):
    return np.ceil(x)


def floor(x):
    return np.floor(x)


def abs(x):  # noqa: A001
    return np.abs(x)


_log_impl = None


def set_log(fn):
    """Substitute the float32 log (the kernels' and the oracle's splat_logf)."""
    global _log_impl
    _log_impl = fn


def log(x):
    return _log_impl(x) if _log_impl is not None else np.log(x)


_exp_impl = None


def set_exp(fn):
    global _exp_impl
    _exp_impl = fn


def exp(x):
    return _exp_impl(x)


def isfinite(x):
    return bool(np.isfinite(x))


def copysign(x, y):
    return F32(np.copysign(np.float32(x), np.float32(y)))


def cross(a, b):
    """wp.cross: (a1 b2 - a2 b1, a2 b0 - a0 b2, a0 b1 - a1 b0)."""
    return a._new([a.v[1] * b.v[2] - a.v[2] * b.v[1], a.v[2] * b.v[0] - a.v[0] * b.v[2],
                   a.v[0] * b.v[1] - a.v[1] * b.v[0]])


def dot(a, b):
    acc = a.v[0] * b.v[0]
    for x, y in zip(a.v[1:], b.v[1:]):
        acc = acc + x * y
    return acc


def length_sq(a):
    return dot(a, a)


def cw_mul(a, b):
    return a._new([x * y for x, y in zip(a.v, b.v)])


def normalize(a):
    """Warp's normalize: a / length(a) per component, zero when length is 0."""
    n = length(a)
    if n > 0:
        return a / n
    return a._new([0.0] * len(a.v))


def outer(a, b):
    out = matrix(len(a.v), len(b.v))()
    for r, x in enumerate(a.v):
        for c, y in enumerate(b.v):
            out.m[r][c] = x * y
    return out


def length(a):
    return sqrt(dot(a, a))


def transpose(m):
    R, C = type(m).rows, type(m).cols
    out = matrix(C, R)()
    for r in range(R):
        for c in range(C):
            out.m[c][r] = m.m[r][c]
    return out


def determinant(m):
    return F32(np.linalg.det(np.array(m.m, np.float64)))


def inverse(m):
    inv = np.linalg.inv(np.array(m.m, np.float64))
    return type(m)(*[F32(v) for v in inv.ravel()])


def atomic_add(arr: Array, *idx_and_value):
    *idx, value = idx_and_value
    key = tuple(idx) if len(idx) > 1 else idx[0]
    with _atomic_lock:
        old = arr.data[key]
        if isinstance(value, Vec):
            arr.data[key] = old + np.array(value.v, dtype=arr.data.dtype)
            return None
        arr.data[key] = old + value
        return old


def static(x):
    return x


def uint64(x):
    return np.uint64(x)


def uint32(x):
    return np.uint32(x) if not isinstance(x, np.uint64) else np.uint32(int(x) & 0xFFFFFFFF)


def float64(x):
    return F64(x)


def grad(f):
    """Gradient of a scalar @wp.func w.r.t. its first (vector) argument by
    central differences in float64 (the kernels call it on `basis`)."""
    src = getattr(f, "__wp_source__", f)

    def g(x, *rest):
        _state.f64 = True
        try:
            base = [F64(v) for v in x.v]
            out = []
            for k in range(len(base)):
                h = 1e-6
                up = list(base); up[k] += h
                dn = list(base); dn[k] -= h
                V = vector(len(base), F64)
                fu = _recompiled_f64(src)(V(*up), *rest)
                fd = _recompiled_f64(src)(V(*dn), *rest)
                out.append((fu - fd) / (2 * h))
        finally:
            _state.f64 = False
        return vector(len(base))(*[F32(v) for v in out]), None
    return g


_f64_cache: dict = {}


def _recompiled_f64(src):
    if src not in _f64_cache:
        _f64_cache[src] = _recompile(src)
    return _f64_cache[src]


def struct(cls):
    fields = dict(getattr(cls, "__annotations__", {}))

    def __init__(self):
        for name, ann in fields.items():
            if isinstance(ann, type) and issubclass(ann, (Vec, Mat)):
                setattr(self, name, ann())
            elif ann is float:
                setattr(self, name, F32(0))
            elif ann is int:
                setattr(self, name, 0)
            elif isinstance(ann, _ArrayType):
                # a default-constructed struct holds null arrays (shape 0)
                setattr(self, name, Array(np.zeros((0,) * max(ann.ndim, 1), np.float32)))
            else:
                setattr(self, name, None)
    return type(cls.__name__, (), {"__init__": __init__, "__annotations__": fields})


def array(*args, dtype=float, ndim=1, **kw):
    return _ArrayType(dtype=dtype, ndim=ndim)


def array2d(*args, dtype=float, **kw):
    return _ArrayType(dtype=dtype, ndim=2)


def array3d(*args, dtype=float, **kw):
    return _ArrayType(dtype=dtype, ndim=3)


def constant(x):
    return x


def _unsupported(*args, **kw):
    raise NotImplementedError("not available in the Warp stand-in")


def make_module() -> types.ModuleType:
    """The `warp` module object to register in sys.modules."""
    _install_block_natives()
    m = types.ModuleType("warp")
    this = sys.modules[__name__]
    for name in ("kernel", "func", "func_native", "func_grad", "struct", "array", "array2d",
                 "array3d", "tid", "static", "min", "max", "clamp", "sqrt", "ceil", "floor",
                 "abs", "log", "exp", "isfinite", "dot", "length", "transpose", "determinant",
                 "inverse", "atomic_add", "uint64", "uint32", "float64", "grad", "constant",
                 "adjoint", "launch", "normalize", "outer", "length_sq", "cw_mul", "copysign",
                 "cross"):
        setattr(m, name, getattr(this, name))
    m.float32 = F32
    m.int32 = np.int32
    m.uint8 = np.uint8
    m.bool = bool
    m.vec2, m.vec3, m.vec4 = vector(2), vector(3), vector(4)
    m.vec2i, m.vec4i = vector(2, int), vector(4, int)
    m.mat22, m.mat33, m.mat44 = matrix(2, 2), matrix(3, 3), matrix(4, 4)
    m.types = types.SimpleNamespace(vector=lambda length, dtype=float: vector(length, dtype),
                                     matrix=lambda shape, dtype=float: matrix(*shape))
    m.Kernel = Kernel
    m.Function = type("Function", (), {})
    m.Stream = type("Stream", (), {})
    m.ScopedStream = _unsupported
    m.utils = types.SimpleNamespace(array_scan=_unsupported, radix_sort_pairs=_unsupported)
    m.init = lambda: None
    m.tile, m.tile_sum, m.launch_tiled = tile, tile_sum, launch_tiled
    m.tile_atomic_add = _unsupported
    m.from_torch = m.get_stream = m.stream_from_torch = _unsupported
    m.device_from_torch = m.dtype_from_torch = _unsupported
    m.config = types.SimpleNamespace()
    return m
