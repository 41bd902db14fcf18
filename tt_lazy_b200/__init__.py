"""tt_lazy on B200: the lazy-tensor front end (C++, ``host/``) over the
sm_100a CUDA backend ``tt_cuda_lib`` (``csrc/``, C-ABI in ``include/tt_cuda.h``).

* ``tt_lazy_b200.capi`` -- ctypes binding of the C-ABI (device pointers in,
  status out), the boundary a C / C++ / FFI caller binds.
* the front end -- ``constant``, ``materialized``, ``relu``, ``sigmoid``,
  ``add``, ``multiply``, ``matmul``, ``transpose``, ``split``,
  ``reduce_sum``, ``reduce_mean``, ``fused_mlp``, ``evaluate``, ``tape``,
  ``stats`` -- re-exported from the pybind11 module over the C++ classes.

Both load in-tree shared objects built by ``python tt_lazy_b200/build.py``;
a missing build is an ImportError, never a CPU fallback.
"""
from . import capi  # noqa: F401

try:
    from . import _tt_lazy as _fe
except ImportError as e:  # pragma: no cover - only before the first build
    raise ImportError(f"tt_lazy_b200 front end not built ({e}); run python tt_lazy_b200/build.py") from e

Tensor = _fe.Tensor
constant = _fe.constant
materialized = _fe.materialized
relu = _fe.relu
sigmoid = _fe.sigmoid
add = _fe.add
multiply = _fe.multiply
matmul = _fe.matmul
transpose = _fe.transpose
split = _fe.split
reduce_sum = _fe.reduce_sum
reduce_mean = _fe.reduce_mean
fused_mlp = _fe.fused_mlp
evaluate = _fe.evaluate
clear = _fe.clear
clear_cache = _fe.clear_cache
tape = _fe.tape
stats = _fe.stats
reset_peak = _fe.reset_peak
graph_size = _fe.graph_size
set_optimization = _fe.set_optimization
synchronize = _fe.synchronize
backend_init = _fe.backend_init
set_gemm_path = _fe.set_gemm_path
streamed = _fe.streamed
all_reduce_sum = _fe.all_reduce_sum
comm_unique_id = _fe.comm_unique_id
comm_init = _fe.comm_init
comm_destroy = _fe.comm_destroy
Plan = _fe.Plan
stream = _fe.stream
set_profiling = _fe.set_profiling
profile = _fe.profile
set_canaries = _fe.set_canaries
check_canaries = _fe.check_canaries
canary_offset = _fe.canary_offset
