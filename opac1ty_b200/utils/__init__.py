from .cuda_kernels import (CudaKernelManager, GPUInfo, MetalKernelManager, get_cuda_device_info,
                           get_metal_device_info)

__all__ = ["CudaKernelManager", "MetalKernelManager", "GPUInfo", "get_cuda_device_info", "get_metal_device_info"]
