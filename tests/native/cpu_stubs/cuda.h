// Host-only stand-in for the CUDA driver types named by vb/symheap.h.
#pragma once
typedef unsigned long long CUdeviceptr;
typedef unsigned long long CUmemGenericAllocationHandle;
