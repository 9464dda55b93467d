"""mambo_b200: B200-native (sm_100a) IQ3_S x MXFP8 quantized-linear path.

Drop-in for Menooker/Mambo's operator API:

    mambo_b200.kernels.quantize_fp8.launch_quantize_fp8
    mambo_b200.kernels.iq3_s_fp8.launch_iq3_s_fp8_matmul / launch_dequant_iq3_s
    mambo_b200.utils.iq3_s_weight.prepare_iq3_s_fields / IQ3SFields
    mambo_b200.utils.kernel_benchmark.BenchmarkCase / mini_benchmark

Arrays are torch CUDA tensors (or any DLPack / __cuda_array_interface__
object). The compute runs in libmambo_b200.so (hand-written sm_100a CUDA);
there is no CPU path.
"""

__version__ = "0.1.0"


def install_as_mambo() -> None:
    """Register this package under the reference's module names (``mambo.kernels.*``, ``mambo.utils.*``).

    Lets code written against the reference import this build unchanged.
    """
    import sys

    from . import kernels, utils
    from .kernels import iq3_s_fp8, quantize_fp8
    from .utils import iq3_s_weight, kernel_benchmark

    pkg = sys.modules[__name__]
    sys.modules.setdefault("mambo", pkg)
    sys.modules["mambo.kernels"] = kernels
    sys.modules["mambo.kernels.iq3_s_fp8"] = iq3_s_fp8
    sys.modules["mambo.kernels.quantize_fp8"] = quantize_fp8
    sys.modules["mambo.utils"] = utils
    sys.modules["mambo.utils.iq3_s_weight"] = iq3_s_weight
    sys.modules["mambo.utils.kernel_benchmark"] = kernel_benchmark
