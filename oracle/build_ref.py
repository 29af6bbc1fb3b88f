"""Builds the reference project's own CUDA megakernels from their sources, for sm_100a, into
oracle/_ref/ — TEST INFRASTRUCTURE ONLY (a GPU cross-check that pins the CPU oracles).

Sources compiled in place (never copied): src/pi05/{binding.cpp, mk6.cu} and
src/molmoact2/{binding.cpp, mk_ma2.cu} of the reference checkout. They are torch extensions; the
reference builds them with torch.utils.cpp_extension.load for sm_120 (src/pi05/hybrid_model.py:
48-52); here the same call targets sm_100a. Outputs (mk_v6_ref*.so, mk_ma2_ref*.so) stay in
oracle/_ref/, which git ignores and which travels to the GPU box with the working tree.
"""
import glob
import importlib.machinery
import importlib.util
import os

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
# The reference checkout: $FA_REFERENCE_ROOT, else a directory named "reference" beside this
# repository (the layout of the build machine); absent on GPU boxes, which use the prebuilt .so files.
REF = os.environ.get("FA_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
KERNELS = {
    "mk_v6_ref": ["src/pi05/binding.cpp", "src/pi05/mk6.cu"],
    "mk_ma2_ref": ["src/molmoact2/binding.cpp", "src/molmoact2/mk_ma2.cu"],
}
FLAGS = ["-O3", "--use_fast_math", "-gencode=arch=compute_100a,code=sm_100a"]


def built(name):
    hits = glob.glob(os.path.join(OUT, name, f"{name}*.so"))
    return hits[0] if hits else None


def build_if_available(verbose=False):
    """Compiles each reference kernel whose sources exist and whose .so is missing."""
    if not os.path.isdir(REF):
        return {}
    from torch.utils.cpp_extension import load
    res = {}
    for name, srcs in KERNELS.items():
        paths = [os.path.join(REF, s) for s in srcs]
        if not all(os.path.exists(p) for p in paths):
            continue
        if built(name):
            res[name] = built(name)
            continue
        bdir = os.path.join(OUT, name)
        os.makedirs(bdir, exist_ok=True)
        os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
        load(name=name, sources=paths, extra_cuda_cflags=FLAGS, build_directory=bdir, verbose=verbose)
        res[name] = built(name)
    return res


def load_ref(name):
    """Imports a prebuilt reference extension (on the GPU box; no sources needed there)."""
    import torch  # noqa: F401  (the extension links against torch)
    so = built(name)
    if not so:
        raise FileNotFoundError(f"{name} not built: run oracle/build_ref.py where the reference sources exist")
    loader = importlib.machinery.ExtensionFileLoader(name, so)
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build_if_available(verbose=True))
