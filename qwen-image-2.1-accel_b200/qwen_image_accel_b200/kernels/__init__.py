"""sm_100a kernels with explicit numerical contracts, behind the reference's op names.

Each module mirrors one module of the reference's `qwen_image_accel.kernels`
package (same function names and argument meaning) and calls the C ABI of
libqia_b200.so. Inputs must be CUDA tensors; there is no CPU path.
"""
