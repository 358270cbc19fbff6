"""The reference's own CUDA kernels, built for sm_100a as a comparison arm --
TEST / BENCH INFRASTRUCTURE ONLY (never imported by the product).

build(ref) compiles, from the reference checkout in place, the pybind11 module
of python/bindings.cpp with the kernels of src/spherical_harmonics/*.cu,
src/tensor_product/*.cu and src/message_passing/*.cu (bindings.cpp names the
namespace `batmobile`, the kernels `batteries`: -Dbatmobile=batteries joins
them).  Outputs go to oracle/_ref/refcuda/ only; the built module travels with
the repository snapshot, so the GPU box needs no reference tree.

load() imports that module under its own name (`_batmobile`) without
registering it in sys.modules, so it cannot shadow this repository's drop-in
module of the same name.

time_pipelines() times, on the current GPU, the two reference pipelines at the
5000-atom workload (CUDA events, L2 flushed before each timed step):
  * README pipeline: fused_sh_tp_simple -> index_add_ (unweighted; the
    reference's benchmarks/benchmark_fused_sh_tp.py:34-61 at N=5000, C=64);
  * weighted unfused chain: normalise -> spherical_harmonics -> x[src] ->
    tensor_product(W) -> index_add_, forward, and its backward through
    tensor_product_backward and spherical_harmonics_backward
    (benchmarks/benchmark_e2e_mace.py:323-350 semantics, fp32).
"""
import importlib.machinery
import importlib.util
import os

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "refcuda")
SOURCES = ["src/spherical_harmonics/spherical_harmonics.cu", "src/spherical_harmonics/spherical_harmonics_backward.cu",
           "src/tensor_product/tensor_product.cu", "src/tensor_product/tensor_product_backward.cu",
           "src/message_passing/fused_message_passing.cu", "src/message_passing/fused_sh_tp.cu"]


def so_path():
    if not os.path.isdir(OUT):
        return None
    for f in os.listdir(OUT):
        if f.startswith("_batmobile") and f.endswith(".so"):
            return os.path.join(OUT, f)
    return None


def build(ref):
    """Compile the reference's module from the checkout at `ref` into oracle/_ref/refcuda/."""
    from torch.utils import cpp_extension
    os.makedirs(OUT, exist_ok=True)
    srcs = [os.path.join(ref, "python", "bindings.cpp")] + [os.path.join(ref, s) for s in SOURCES]
    cpp_extension.load(
        name="_batmobile", sources=srcs, build_directory=OUT, verbose=False,
        extra_include_paths=[os.path.join(ref, "include")],
        extra_cflags=["-O3", "-Dbatmobile=batteries"],
        extra_cuda_cflags=["-O3", "-Dbatmobile=batteries", "-gencode", "arch=compute_100a,code=sm_100a",
                           "-lineinfo"])
    return so_path()


def load():
    path = so_path()
    if path is None:
        return None
    import torch  # noqa: F401  (the module links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader("_batmobile", path)
    spec = importlib.util.spec_from_file_location("_batmobile", path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def _timed(fn, steps, warmup, flush):
    import torch
    tot = 0.0
    for i in range(warmup + steps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        if i >= warmup:
            tot += s.elapsed_time(e)
    return tot / steps


def time_pipelines(x, vec, W, G, ei, n, steps=5, warmup=2):
    """ms per step of the reference's pipelines on the given device tensors
    (x [N,C,16], vec [E,3] raw edge vectors, W [34,C,C], G [N,C,16], ei [2,E])."""
    import torch
    mod = load()
    if mod is None:
        return {"unavailable": "oracle/_ref/refcuda not built (needs the reference checkout at build time)"}
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=x.device)
    src, dst = ei[0].contiguous(), ei[1].contiguous()
    E = src.numel()
    vhat = vec / vec.norm(dim=1, keepdim=True).clamp(min=1e-8)

    def simple():
        msg = mod.fused_sh_tp_simple(vhat, x, src)
        out = torch.zeros_like(x)
        out.index_add_(0, dst, msg)
        return out

    def weighted_fwd():
        Y = mod.spherical_harmonics(vhat, 3)
        msg = mod.tensor_product(x[src].contiguous(), Y, W)
        out = torch.zeros(n, W.shape[2], 16, device=x.device)
        out.index_add_(0, dst, msg)
        return out

    def weighted_fwd_bwd():
        Y = mod.spherical_harmonics(vhat, 3)
        xs = x[src].contiguous()
        msg = mod.tensor_product(xs, Y, W)
        out = torch.zeros(n, W.shape[2], 16, device=x.device)
        out.index_add_(0, dst, msg)
        gxs, gY, gW = mod.tensor_product_backward(xs, Y, W, G[dst].contiguous(), True, True, True)
        gx = torch.zeros_like(x).index_add_(0, src, gxs)
        gv = mod.spherical_harmonics_backward(vhat, gY)
        return out, gx, gW, gv

    res = {"edges": E, "what": "reference CUDA kernels (python/bindings.cpp + src/*.cu) compiled for sm_100a, "
                               "torch index_add_ scatter; CUDA events, L2 flushed before each step"}
    ms = _timed(simple, steps, warmup, flush)
    res["fused_sh_tp_simple+index_add"] = {"ms": ms, "Medges/s": E / (ms * 1e-3) / 1e6,
                                           "note": "unweighted TP (the reference README's fused pipeline)"}
    ms = _timed(weighted_fwd, steps, warmup, flush)
    res["weighted_forward"] = {"ms": ms, "Medges/s": E / (ms * 1e-3) / 1e6,
                               "note": "SH -> tensor_product(W) on gathered x -> index_add_"}
    ms = _timed(weighted_fwd_bwd, max(1, steps // 2), 1, flush)
    res["weighted_forward_backward"] = {
        "ms": ms, "Medges/s": E / (ms * 1e-3) / 1e6,
        "note": "forward + tensor_product_backward (x, Y, W) + spherical_harmonics_backward; the edge-vector "
                "normalisation's chain rule and the neighbour list are not included"}
    return res
