/*
 * Minimal OpenCL declarations so that the reference's CPU attention sources
 * (compute/attention-gqa-resident/attention_gqa_benchmark.c and
 * compute/gguf-real-weights-loader/test_28_layers_real.c) compile on a machine
 * without OpenCL headers.
 *
 * Test infrastructure only: the oracle build compiles those files with
 * `-Dmain=...` and links with a version script plus --gc-sections, so the
 * OpenCL host code (their main()) is discarded and none of the functions
 * declared below is ever referenced by the resulting library.  Nothing here is
 * defined; the typedefs are opaque.
 */
#ifndef GQA_ORACLE_CL_STUB_H
#define GQA_ORACLE_CL_STUB_H

#include <stddef.h>
#include <stdint.h>

typedef int32_t  cl_int;
typedef uint32_t cl_uint;
typedef uint64_t cl_ulong;
typedef cl_uint  cl_bool;
typedef cl_ulong cl_bitfield;
typedef cl_bitfield cl_device_type;
typedef cl_bitfield cl_mem_flags;
typedef cl_bitfield cl_command_queue_properties;
typedef cl_uint cl_device_info;
typedef cl_uint cl_program_build_info;
typedef cl_uint cl_buffer_create_type;
typedef intptr_t cl_context_properties;

typedef struct gqa_stub_platform *cl_platform_id;
typedef struct gqa_stub_device *cl_device_id;
typedef struct gqa_stub_context *cl_context;
typedef struct gqa_stub_queue *cl_command_queue;
typedef struct gqa_stub_program *cl_program;
typedef struct gqa_stub_kernel *cl_kernel;
typedef struct gqa_stub_mem *cl_mem;
typedef struct gqa_stub_event *cl_event;

typedef struct { size_t origin; size_t size; } cl_buffer_region;

#define CL_SUCCESS 0
#define CL_FALSE 0
#define CL_TRUE 1
#define CL_DEVICE_TYPE_GPU (1 << 2)
#define CL_DEVICE_NAME 0x102B
#define CL_QUEUE_PROFILING_ENABLE (1 << 1)
#define CL_PROGRAM_BUILD_LOG 0x1183
#define CL_MEM_READ_WRITE (1 << 0)
#define CL_MEM_READ_ONLY (1 << 2)
#define CL_MEM_COPY_HOST_PTR (1 << 5)
#define CL_BUFFER_CREATE_TYPE_REGION 0x1220

cl_int clGetPlatformIDs(cl_uint, cl_platform_id *, cl_uint *);
cl_int clGetDeviceIDs(cl_platform_id, cl_device_type, cl_uint, cl_device_id *, cl_uint *);
cl_int clGetDeviceInfo(cl_device_id, cl_device_info, size_t, void *, size_t *);
cl_context clCreateContext(const cl_context_properties *, cl_uint, const cl_device_id *,
                           void (*)(const char *, const void *, size_t, void *), void *, cl_int *);
cl_command_queue clCreateCommandQueue(cl_context, cl_device_id, cl_command_queue_properties, cl_int *);
cl_program clCreateProgramWithSource(cl_context, cl_uint, const char **, const size_t *, cl_int *);
cl_int clBuildProgram(cl_program, cl_uint, const cl_device_id *, const char *,
                      void (*)(cl_program, void *), void *);
cl_int clGetProgramBuildInfo(cl_program, cl_device_id, cl_program_build_info, size_t, void *, size_t *);
cl_kernel clCreateKernel(cl_program, const char *, cl_int *);
cl_mem clCreateBuffer(cl_context, cl_mem_flags, size_t, void *, cl_int *);
cl_mem clCreateSubBuffer(cl_mem, cl_mem_flags, cl_buffer_create_type, const void *, cl_int *);
cl_int clSetKernelArg(cl_kernel, cl_uint, size_t, const void *);
cl_int clEnqueueNDRangeKernel(cl_command_queue, cl_kernel, cl_uint, const size_t *, const size_t *,
                              const size_t *, cl_uint, const cl_event *, cl_event *);
cl_int clEnqueueWriteBuffer(cl_command_queue, cl_mem, cl_bool, size_t, size_t, const void *,
                            cl_uint, const cl_event *, cl_event *);
cl_int clEnqueueReadBuffer(cl_command_queue, cl_mem, cl_bool, size_t, size_t, void *,
                           cl_uint, const cl_event *, cl_event *);
cl_int clEnqueueFillBuffer(cl_command_queue, cl_mem, const void *, size_t, size_t, size_t,
                           cl_uint, const cl_event *, cl_event *);
cl_int clFinish(cl_command_queue);
cl_int clWaitForEvents(cl_uint, const cl_event *);
cl_int clReleaseEvent(cl_event);
cl_int clReleaseMemObject(cl_mem);
cl_int clReleaseKernel(cl_kernel);
cl_int clReleaseProgram(cl_program);
cl_int clReleaseCommandQueue(cl_command_queue);
cl_int clReleaseContext(cl_context);

#endif
