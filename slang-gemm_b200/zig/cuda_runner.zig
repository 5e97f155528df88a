//! cuda_runner.zig -- slang-gemm's GPU runner on NVIDIA B200 (sm_100a): the drop-in replacement of
//! src/vulkan_runner.zig, built on libgemm_sm100 (include/gemm_sm100.h, through @cImport).
//!
//! bench/gemm_perf.zig times its shader column through eleven `vulkan_runner.bench*Case` functions
//! (call sites :337, :415, :474, :551, :639, :644, :649, :655, :777, :782, :788, :845, :920, :996) and
//! reads `vulkan_runner.Result` (:38). This file exports every public `bench*` function of
//! src/vulkan_runner.zig with the same name and parameter list, and the same `Result`
//! (src/vulkan_runner.zig:18-21), so the unmodified bench compiles against it once the `vulkan_runner`
//! module is built from this file (BUILD.bazel: `main = "src/cuda_runner.zig"`).
//!
//! Each case fills its operands with the Vulkan runner's deterministic patterns
//! (src/vulkan_runner.zig:2221-2288: biases 0.1 / -0.2, INT8 1 / -2), zeroes C, makes `warmup` untimed
//! calls, then times `iters` calls between two CUDA events, and returns milliseconds per call and
//! TFLOP/s as 2*m*n*k*batch_count / ms (bench/gemm_perf.zig:1279-1282). Operands are column-major
//! with tight leading dimensions, the cuBLAS convention the bench's cuBLAS column uses.
//!
//! Which library path each case takes:
//!   FP32 sgemm (benchSgemmF32*, benchNvcoop2F32*)          -> FFMA kernel, exact f32 products
//!   FP16 / BF16 -> FP32 (benchNvcoop2F16*, Bf16*, LowpF32*) -> tcgen05 kind::f16, f32 accumulate
//!   FP16 -> FP16 (benchF16ScalarCase)                       -> tcgen05 kind::f16, f16 output
//!   INT8 -> INT32 (benchInt8I32*, benchNvcoop2I8*)         -> tcgen05 kind::i8, exact s32
//!   FP64, complex, FP8 / FP6 / FP4 (benchDgemm*, benchCgemm*, benchZgemm*, other LowpF32 types)
//!                                                           -> null: no kernel in this backend
//!
//! Return conventions are vulkan_runner.zig's:
//!   - `null` when this backend has no kernel for the case, or the chosen device is not compute
//!     capability 10.0; the bench then reports the shader column as unavailable.
//!   - error.NoVulkanDevice when there is no CUDA device at all; error.NoMatchingDevice when no device
//!     name contains `device_substr` (selectPhysicalDevice, src/vulkan_runner.zig:1273-1299). The
//!     bench's catch switches (e.g. bench/gemm_perf.zig:337-339) also name error.TimestampUnsupported
//!     and error.VulkanFailure, so both belong to `Error`; this runner never returns them (CUDA events
//!     always time, and there is no Vulkan).
//!   - error.InvalidArgument for an empty shape, zero iterations or a dimension beyond a C int
//!     (src/vulkan_runner.zig:223-225).
//!   - error.CudaGemmFailure when the library returns a failure status, or when a kernel's bounded
//!     pipeline wait gave up (gs_device_error); the bench propagates it (`else => return err`).
//!
//! Two CUDA runtimes meet in one process: libgemm_sm100 links its own (static) cudart and the
//! reference's src/cublas.zig links libcudart. Both work in the device's primary context and its
//! legacy default stream, so device buffers from cublas.RawDeviceBuffer, the library's kernels and
//! cublas.GpuTimer's events all see the same memory and the same stream; the selected device is made
//! current in both runtimes.
const std = @import("std");
const gemm = @import("gemm");
const cublas = @import("cublas");
const c = @cImport(@cInclude("gemm_sm100.h"));

extern fn cudaSetDevice(device: c_int) callconv(.c) c_int;
extern fn cudaMemset(ptr: ?*anyopaque, value: c_int, count: usize) callconv(.c) c_int;

pub const Result = struct {
    ms: f64,
    tflops: f64,
};

/// Errors of every bench* function (see the file comment for when each is returned).
pub const Error = error{
    NoVulkanDevice,
    NoMatchingDevice,
    TimestampUnsupported,
    VulkanFailure,
    InvalidArgument,
    CudaGemmFailure,
    CudaFailure,
    BufferTooSmall,
    OutOfMemory,
};

/// Operand element type of a case.
const In = enum { f32, f16, bf16, i8 };
/// Output element type of a case.
const Out = enum { f32, f16, i32 };

fn inBytes(t: In) usize {
    return switch (t) {
        .f32 => 4,
        .f16, .bf16 => 2,
        .i8 => 1,
    };
}

fn outBytes(t: Out) usize {
    return switch (t) {
        .f16 => 2,
        .f32, .i32 => 4,
    };
}

fn inType(t: In) c_int {
    return switch (t) {
        .f32 => c.GS_R_32F,
        .f16 => c.GS_R_16F,
        .bf16 => c.GS_R_16BF,
        .i8 => c.GS_R_8I,
    };
}

fn outType(t: Out) c_int {
    return switch (t) {
        .f32 => c.GS_R_32F,
        .f16 => c.GS_R_16F,
        .i32 => c.GS_R_32I,
    };
}

fn opValue(op: gemm.Op) c_int {
    return switch (op) {
        .no_trans => c.GS_OP_N,
        .trans => c.GS_OP_T,
        .conj_trans => c.GS_OP_C,
    };
}

fn check(status: anytype) Error!void {
    if (status != 0) return error.CudaGemmFailure;
}

fn tflops(m: usize, n: usize, k: usize, ms: f64) f64 {
    const ops = 2.0 * @as(f64, @floatFromInt(m)) * @as(f64, @floatFromInt(n)) * @as(f64, @floatFromInt(k));
    return ops / (ms * 1.0e9);
}

/// The Vulkan runner's floating-point fill: ((i*19 + 7) % 23 - 11) / 7 + bias.
fn patternF(i: usize, bias: f32) f32 {
    const raw: f32 = @floatFromInt((i * 19 + 7) % 23);
    return (raw - 11) / 7 + bias;
}

/// The Vulkan runner's INT8 fill: (i*7 + 3) % 17 - 8 + bias.
fn patternI8(i: usize, bias: i32) i8 {
    const raw: i32 = @intCast((i * 7 + 3) % 17);
    return @intCast(raw - 8 + bias);
}

/// Allocates a device buffer of `count` elements of type `t` and uploads the fill pattern with `bias`
/// (INT8 operands use `ibias`).
fn upload(allocator: std.mem.Allocator, t: In, count: usize, bias: f32, ibias: i32) Error!cublas.RawDeviceBuffer {
    const buf = try cublas.RawDeviceBuffer.alloc(count * inBytes(t));
    errdefer buf.free();
    switch (t) {
        .f32 => {
            const v = try allocator.alloc(f32, count);
            defer allocator.free(v);
            for (v, 0..) |*x, i| x.* = patternF(i, bias);
            try buf.copyFromHost(std.mem.sliceAsBytes(v));
        },
        .f16, .bf16 => {
            const v = try allocator.alloc(u16, count);
            defer allocator.free(v);
            for (v, 0..) |*x, i| x.* = if (t == .f16) gemm.f32ToF16Bits(patternF(i, bias)) else gemm.f32ToBf16Bits(patternF(i, bias));
            try buf.copyFromHost(std.mem.sliceAsBytes(v));
        },
        .i8 => {
            const v = try allocator.alloc(i8, count);
            defer allocator.free(v);
            for (v, 0..) |*x, i| x.* = patternI8(i, ibias);
            try buf.copyFromHost(std.mem.sliceAsBytes(v));
        },
    }
    return buf;
}

/// Makes the first CUDA device whose name contains `device_substr` current in both CUDA runtimes.
/// Returns false when the matching devices are not compute capability 10.0 (no kernel here).
fn selectDevice(allocator: std.mem.Allocator, device_substr: ?[]const u8) Error!bool {
    var dev: c_int = -1;
    const status = if (device_substr) |needle| blk: {
        const z = try allocator.dupeZ(u8, needle);
        defer allocator.free(z);
        break :blk c.gs_select_device(z.ptr, &dev);
    } else c.gs_select_device(null, &dev);
    if (status == c.GS_STATUS_NOT_INITIALIZED) return error.NoVulkanDevice;
    if (status == c.GS_STATUS_INVALID_VALUE) return error.NoMatchingDevice;
    if (status != c.GS_STATUS_SUCCESS) return false;
    if (cudaSetDevice(dev) != 0) return error.CudaFailure;
    return true;
}

/// The arguments of one gs_gemm_strided_batched_ex call (alpha = 1, beta = 0, ldc = m).
const Call = struct {
    handle: c.gs_handle,
    op_a: c_int,
    op_b: c_int,
    m: c_int,
    n: c_int,
    k: c_int,
    alpha: ?*const anyopaque,
    beta: ?*const anyopaque,
    a: ?*anyopaque,
    b: ?*anyopaque,
    cc: ?*anyopaque,
    in_type: c_int,
    out_type: c_int,
    lda: c_int,
    ldb: c_int,
    stride_a: c_longlong,
    stride_b: c_longlong,
    stride_c: c_longlong,
    batch: c_int,
    compute: c_int,

    fn run(self: Call) Error!void {
        try check(c.gs_gemm_strided_batched_ex(self.handle, self.op_a, self.op_b, self.m, self.n, self.k,
            self.alpha, self.a, self.in_type, self.lda, self.stride_a, self.b, self.in_type, self.ldb,
            self.stride_b, self.beta, self.cc, self.out_type, self.m, self.stride_c, self.batch, self.compute,
            c.GS_GEMM_DEFAULT));
    }
};

/// One timed case: C = op(A) op(B) over `batch_count` strided entries (strides of one extent),
/// alpha = 1, beta = 0, through gs_gemm_strided_batched_ex.
fn timeCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, in: In, out: Out, m: usize, n: usize,
            k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    if (m == 0 or n == 0 or k == 0 or batch_count == 0 or iters == 0) return error.InvalidArgument;
    const limit: usize = std.math.maxInt(c_int);
    if (m > limit or n > limit or k > limit or batch_count > limit) return error.InvalidArgument;
    if (!try selectDevice(allocator, device_substr)) return null;

    var handle: c.gs_handle = null;
    if (c.gs_create(&handle) != c.GS_STATUS_SUCCESS) return null;
    defer _ = c.gs_destroy(handle);

    const a_rows = gemm.storedRows(op_a, m, k);
    const a_len = a_rows * gemm.storedCols(op_a, m, k);
    const b_rows = gemm.storedRows(op_b, k, n);
    const b_len = b_rows * gemm.storedCols(op_b, k, n);
    const c_len = m * n;
    const da = try upload(allocator, in, a_len * batch_count, 0.1, 1);
    defer da.free();
    const db = try upload(allocator, in, b_len * batch_count, -0.2, -2);
    defer db.free();
    const c_bytes = c_len * batch_count * outBytes(out);
    const dc = try cublas.RawDeviceBuffer.alloc(c_bytes);
    defer dc.free();
    if (cudaMemset(dc.ptr, 0, c_bytes) != 0) return error.CudaFailure;

    const f_one: f32 = 1;
    const f_zero: f32 = 0;
    const i_one: i32 = 1;
    const i_zero: i32 = 0;
    const integer = in == .i8;
    const call = Call{
        .handle = handle,
        .op_a = opValue(op_a),
        .op_b = opValue(op_b),
        .m = @intCast(m),
        .n = @intCast(n),
        .k = @intCast(k),
        .alpha = if (integer) @ptrCast(&i_one) else @ptrCast(&f_one),
        .beta = if (integer) @ptrCast(&i_zero) else @ptrCast(&f_zero),
        .a = da.ptr,
        .b = db.ptr,
        .cc = dc.ptr,
        .in_type = inType(in),
        .out_type = outType(out),
        .lda = @intCast(a_rows),
        .ldb = @intCast(b_rows),
        .stride_a = @intCast(a_len),
        .stride_b = @intCast(b_len),
        .stride_c = @intCast(c_len),
        .batch = @intCast(batch_count),
        .compute = if (integer) c.GS_COMPUTE_32I else c.GS_COMPUTE_32F,
    };
    var i: usize = 0;
    while (i < warmup) : (i += 1) try call.run();
    try cublas.synchronize();
    const timer = try cublas.GpuTimer.init();
    defer timer.deinit();
    try timer.begin();
    i = 0;
    while (i < iters) : (i += 1) try call.run();
    const total_ms = try timer.end();
    var word: u32 = 0;
    try check(c.gs_device_error(handle, &word));
    if (word != 0) return error.CudaGemmFailure;
    const ms = @as(f64, total_ms) / @as(f64, @floatFromInt(iters));
    return .{ .ms = ms, .tflops = tflops(m, n, k, ms) * @as(f64, @floatFromInt(batch_count)) };
}

/// FP16 / BF16 operand types of the low-precision cases; any other type has no kernel here.
fn lowpIn(a_type: gemm.DataType, b_type: gemm.DataType) ?In {
    if (a_type != b_type) return null;
    return switch (a_type) {
        .r_16f => .f16,
        .r_16bf => .bf16,
        else => null,
    };
}

// ---- FP32 -------------------------------------------------------------------------------------------

pub fn benchSgemmF32(allocator: std.mem.Allocator, size: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchSgemmF32Case(allocator, .no_trans, .no_trans, size, size, size, iters, warmup, device_substr);
}

pub fn benchSgemmF32Case(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchSgemmF32BatchedCase(allocator, op_a, op_b, m, n, k, 1, iters, warmup, device_substr);
}

pub fn benchSgemmF32BatchedCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return timeCase(allocator, op_a, op_b, .f32, .f32, m, n, k, batch_count, iters, warmup, device_substr);
}

/// The Vulkan runner's FP32 cooperative-matrix candidate: here the same exact FFMA kernel.
pub fn benchNvcoop2F32StridedBatchedOpCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return timeCase(allocator, op_a, op_b, .f32, .f32, m, n, k, batch_count, iters, warmup, device_substr);
}

// ---- FP64 and complex: no kernel in this backend -------------------------------------------------------

fn unavailable(allocator: std.mem.Allocator, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, device_substr: ?[]const u8) Error!?Result {
    if (m == 0 or n == 0 or k == 0 or batch_count == 0 or iters == 0) return error.InvalidArgument;
    _ = try selectDevice(allocator, device_substr);
    return null;
}

pub fn benchDgemmF64Case(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchDgemmF64BatchedCase(allocator, op_a, op_b, m, n, k, 1, iters, warmup, device_substr);
}

pub fn benchDgemmF64BatchedCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    _ = op_a;
    _ = op_b;
    _ = warmup;
    return unavailable(allocator, m, n, k, batch_count, iters, device_substr);
}

pub fn benchCgemmF32Case(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchCgemmF32BatchedCase(allocator, op_a, op_b, m, n, k, 1, iters, warmup, device_substr);
}

pub fn benchCgemmF32BatchedCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    _ = op_a;
    _ = op_b;
    _ = warmup;
    return unavailable(allocator, m, n, k, batch_count, iters, device_substr);
}

pub fn benchZgemmF64Case(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchZgemmF64BatchedCase(allocator, op_a, op_b, m, n, k, 1, iters, warmup, device_substr);
}

pub fn benchZgemmF64BatchedCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    _ = op_a;
    _ = op_b;
    _ = warmup;
    return unavailable(allocator, m, n, k, batch_count, iters, device_substr);
}

// ---- FP16 / BF16 -> FP32 on the tensor cores ------------------------------------------------------------

pub fn benchLowpF32Case(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, a_type: gemm.DataType, b_type: gemm.DataType, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchLowpF32BatchedCase(allocator, op_a, op_b, a_type, b_type, m, n, k, 1, iters, warmup, device_substr);
}

/// The Vulkan runner's decode-then-FFMA fallback for FP16/BF16/FP8/FP6/FP4 -> FP32: FP16 and BF16 run on
/// the tensor cores here; the other types have no kernel in this backend.
pub fn benchLowpF32BatchedCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, a_type: gemm.DataType, b_type: gemm.DataType, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    const in = lowpIn(a_type, b_type) orelse return unavailable(allocator, m, n, k, batch_count, iters, device_substr);
    return timeCase(allocator, op_a, op_b, in, .f32, m, n, k, batch_count, iters, warmup, device_substr);
}

pub fn benchNvcoop2F16Case(allocator: std.mem.Allocator, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchNvcoop2F16StridedBatchedOpCase(allocator, .no_trans, .no_trans, m, n, k, 1, iters, warmup, device_substr);
}

pub fn benchNvcoop2F16SmallCase(allocator: std.mem.Allocator, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchNvcoop2F16StridedBatchedOpCase(allocator, .no_trans, .no_trans, m, n, k, 1, iters, warmup, device_substr);
}

pub fn benchNvcoop2F16StridedBatchedCase(allocator: std.mem.Allocator, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchNvcoop2F16StridedBatchedOpCase(allocator, .no_trans, .no_trans, m, n, k, batch_count, iters, warmup, device_substr);
}

pub fn benchNvcoop2F16StridedBatchedOpCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return timeCase(allocator, op_a, op_b, .f16, .f32, m, n, k, batch_count, iters, warmup, device_substr);
}

pub fn benchNvcoop2Bf16Case(allocator: std.mem.Allocator, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchNvcoop2Bf16StridedBatchedOpCase(allocator, .no_trans, .no_trans, m, n, k, 1, iters, warmup, device_substr);
}

pub fn benchNvcoop2Bf16StridedBatchedCase(allocator: std.mem.Allocator, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchNvcoop2Bf16StridedBatchedOpCase(allocator, .no_trans, .no_trans, m, n, k, batch_count, iters, warmup, device_substr);
}

pub fn benchNvcoop2Bf16StridedBatchedOpCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return timeCase(allocator, op_a, op_b, .bf16, .f32, m, n, k, batch_count, iters, warmup, device_substr);
}

// ---- FP16 -> FP16 ---------------------------------------------------------------------------------------

/// The Vulkan runner's scalar FP16 shader (shaders/gemm_real_f16.slang): here the tensor-core kernel
/// with f32 accumulation and an FP16 output.
pub fn benchF16ScalarCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return timeCase(allocator, op_a, op_b, .f16, .f16, m, n, k, batch_count, iters, warmup, device_substr);
}

// ---- INT8 -> INT32 on the tensor cores ------------------------------------------------------------------

pub fn benchInt8I32Case(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchInt8I32BatchedCase(allocator, op_a, op_b, m, n, k, 1, iters, warmup, device_substr);
}

pub fn benchInt8I32BatchedCase(allocator: std.mem.Allocator, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return timeCase(allocator, op_a, op_b, .i8, .i32, m, n, k, batch_count, iters, warmup, device_substr);
}

pub fn benchNvcoop2I8Case(allocator: std.mem.Allocator, m: usize, n: usize, k: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchInt8I32BatchedCase(allocator, .no_trans, .no_trans, m, n, k, 1, iters, warmup, device_substr);
}

pub fn benchNvcoop2I8StridedBatchedCase(allocator: std.mem.Allocator, m: usize, n: usize, k: usize, batch_count: usize, iters: usize, warmup: usize, device_substr: ?[]const u8) Error!?Result {
    return benchInt8I32BatchedCase(allocator, .no_trans, .no_trans, m, n, k, batch_count, iters, warmup, device_substr);
}

// ---- library calls: the src/cublas.zig counterparts on libgemm_sm100 ----------------------------------
// Same names and arguments as cublas.zig's (Context :78-90, sgemm :171-173, sgemmStridedBatched :195-197,
// sgemmBatched :211-213, gemmEx :227-229, gemmStridedBatchedEx :235-237, gemmBatchedEx :239-241), so a
// caller switches backends by switching the import. Errors: error.CudaGemmFailure for any non-success
// status (cublas.zig's checkCublas maps to error.CublasFailure, :73-76).

/// cublas.Context counterpart: one libgemm_sm100 handle on the current device and the legacy default
/// stream. Not thread-safe; use one per host thread.
pub const Context = struct {
    handle: c.gs_handle,

    pub fn init() Error!Context {
        var h: c.gs_handle = null;
        try check(c.gs_create(&h));
        return .{ .handle = h };
    }

    pub fn deinit(self: Context) void {
        _ = c.gs_destroy(self.handle);
    }

    /// Orders this context's calls on `stream` (a cudaStream_t; null is the legacy default stream).
    pub fn setStream(self: Context, stream: ?*anyopaque) Error!void {
        try check(c.gs_set_stream(self.handle, stream));
    }
};

fn int(value: usize) c_int {
    return @intCast(value);
}

fn long(value: usize) c_longlong {
    return @intCast(value);
}

pub fn sgemm(ctx: Context, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, alpha: f32, a: [*]const f32, lda: usize, b: [*]const f32, ldb: usize, beta: f32, cc: [*]f32, ldc: usize) Error!void {
    try check(c.gs_sgemm(ctx.handle, opValue(op_a), opValue(op_b), int(m), int(n), int(k), &alpha, a, int(lda), b,
        int(ldb), &beta, cc, int(ldc)));
}

pub fn sgemmStridedBatched(ctx: Context, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, alpha: f32, a: [*]const f32, lda: usize, stride_a: usize, b: [*]const f32, ldb: usize, stride_b: usize, beta: f32, cc: [*]f32, ldc: usize, stride_c: usize, batch_count: usize) Error!void {
    try check(c.gs_sgemm_strided_batched(ctx.handle, opValue(op_a), opValue(op_b), int(m), int(n), int(k), &alpha,
        a, int(lda), long(stride_a), b, int(ldb), long(stride_b), &beta, cc, int(ldc), long(stride_c),
        int(batch_count)));
}

/// FP32 pointer-array batch: the arrays are device memory holding device pointers, as with cuBLAS.
pub fn sgemmBatched(ctx: Context, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, alpha: f32, a_array: ?*const anyopaque, lda: usize, b_array: ?*const anyopaque, ldb: usize, beta: f32, c_array: ?*anyopaque, ldc: usize, batch_count: usize) Error!void {
    try check(c.gs_gemm_batched_ex(ctx.handle, opValue(op_a), opValue(op_b), int(m), int(n), int(k), &alpha,
        @ptrCast(@alignCast(a_array)), c.GS_R_32F, int(lda), @ptrCast(@alignCast(b_array)), c.GS_R_32F, int(ldb),
        &beta, @ptrCast(@alignCast(c_array)), c.GS_R_32F, int(ldc), int(batch_count), c.GS_COMPUTE_32F,
        c.GS_GEMM_DEFAULT));
}

/// gemm.hgemm (src/gemm.zig:438-477) on the device: f16 bits in and out, f16 alpha / beta bits,
/// f32 accumulation.
pub fn hgemm(ctx: Context, op_a: gemm.Op, op_b: gemm.Op, m: usize, n: usize, k: usize, alpha_bits: u16, a: [*]const u16, lda: usize, b: [*]const u16, ldb: usize, beta_bits: u16, cc: [*]u16, ldc: usize) Error!void {
    try check(c.gs_hgemm(ctx.handle, opValue(op_a), opValue(op_b), int(m), int(n), int(k), &alpha_bits, a,
        int(lda), b, int(ldb), &beta_bits, cc, int(ldc)));
}

pub fn gemmEx(ctx: Context, desc: cublas.RawGemmExDesc) Error!void {
    try check(c.gs_gemm_ex(ctx.handle, opValue(desc.op_a), opValue(desc.op_b), int(desc.m), int(desc.n),
        int(desc.k), desc.alpha, desc.a, @intFromEnum(desc.a_type), int(desc.lda), desc.b,
        @intFromEnum(desc.b_type), int(desc.ldb), desc.beta, desc.c, @intFromEnum(desc.c_type), int(desc.ldc),
        @intFromEnum(desc.compute_type), @intFromEnum(desc.algo)));
}

pub fn gemmStridedBatchedEx(ctx: Context, desc: cublas.RawGemmExDesc) Error!void {
    try check(c.gs_gemm_strided_batched_ex(ctx.handle, opValue(desc.op_a), opValue(desc.op_b), int(desc.m),
        int(desc.n), int(desc.k), desc.alpha, desc.a, @intFromEnum(desc.a_type), int(desc.lda),
        long(desc.stride_a), desc.b, @intFromEnum(desc.b_type), int(desc.ldb), long(desc.stride_b), desc.beta,
        desc.c, @intFromEnum(desc.c_type), int(desc.ldc), long(desc.stride_c), int(desc.batch_count),
        @intFromEnum(desc.compute_type), @intFromEnum(desc.algo)));
}

pub fn gemmBatchedEx(ctx: Context, desc: cublas.RawGemmBatchedExDesc) Error!void {
    try check(c.gs_gemm_batched_ex(ctx.handle, opValue(desc.op_a), opValue(desc.op_b), int(desc.m), int(desc.n),
        int(desc.k), desc.alpha, @ptrCast(@alignCast(desc.a_array)), @intFromEnum(desc.a_type), int(desc.lda),
        @ptrCast(@alignCast(desc.b_array)), @intFromEnum(desc.b_type), int(desc.ldb), desc.beta,
        @ptrCast(@alignCast(desc.c_array)), @intFromEnum(desc.c_type), int(desc.ldc), int(desc.batch_count),
        @intFromEnum(desc.compute_type), @intFromEnum(desc.algo)));
}

// ---- host-buffer calls: gemm.gemmEx / gemm.gemmBatchedEx on the GPU --------------------------------------

/// gemm.gemmEx / gemm.gemmStridedBatchedEx (src/gemm.zig:546, :632) over the same host ExDesc: A and B (and
/// C when it is read) are copied to the device, computed, and C is copied back before the call returns.
/// Same validation and error meaning as the reference (a failed validation is error.CudaGemmFailure).
pub fn hostGemmEx(ctx: Context, d: gemm.ExDesc) Error!void {
    var x = c.gs_ex_desc{
        .op_a = opValue(d.op_a),
        .op_b = opValue(d.op_b),
        .m = d.m,
        .n = d.n,
        .k = d.k,
        .alpha_re = d.alpha.re,
        .alpha_im = d.alpha.im,
        .a = d.a.ptr,
        .a_len = d.a.len,
        .a_type = @intFromEnum(d.a_type),
        .lda = d.lda,
        .b = d.b.ptr,
        .b_len = d.b.len,
        .b_type = @intFromEnum(d.b_type),
        .ldb = d.ldb,
        .beta_re = d.beta.re,
        .beta_im = d.beta.im,
        .c = d.c.ptr,
        .c_len = d.c.len,
        .c_type = @intFromEnum(d.c_type),
        .ldc = d.ldc,
        .compute_type = @intFromEnum(d.compute_type),
        .layout = if (d.layout == .row_major) c.GS_LAYOUT_ROW_MAJOR else c.GS_LAYOUT_COL_MAJOR,
        .batch_count = d.batch_count,
        .stride_a = d.stride_a,
        .stride_b = d.stride_b,
        .stride_c = d.stride_c,
        .algo = @intFromEnum(d.algo),
    };
    try check(c.gs_host_gemm_ex(ctx.handle, &x));
}

/// gemm.gemmBatchedEx (src/gemm.zig:636-663) over the same PointerBatchedExDesc of host slices. As in the
/// reference's entry-by-entry loop, entries before one that fails validation are computed and written back.
pub fn hostGemmBatchedEx(ctx: Context, allocator: std.mem.Allocator, d: gemm.PointerBatchedExDesc) Error!void {
    const total = d.a.len + d.b.len + d.c.len;
    const ptrs = try allocator.alloc(?*const anyopaque, total);
    defer allocator.free(ptrs);
    const cptrs = try allocator.alloc(?*anyopaque, d.c.len);
    defer allocator.free(cptrs);
    const lens = try allocator.alloc(usize, total);
    defer allocator.free(lens);
    for (d.a, 0..) |s, i| {
        ptrs[i] = s.ptr;
        lens[i] = s.len;
    }
    for (d.b, 0..) |s, i| {
        ptrs[d.a.len + i] = s.ptr;
        lens[d.a.len + i] = s.len;
    }
    const cb = d.a.len + d.b.len;
    for (d.c, 0..) |s, i| {
        cptrs[i] = s.ptr;
        lens[cb + i] = s.len;
    }
    var x = c.gs_ptr_batched_desc{
        .op_a = opValue(d.op_a),
        .op_b = opValue(d.op_b),
        .m = d.m,
        .n = d.n,
        .k = d.k,
        .alpha_re = d.alpha.re,
        .alpha_im = d.alpha.im,
        .a = ptrs.ptr,
        .a_lens = lens.ptr,
        .a_count = d.a.len,
        .a_type = @intFromEnum(d.a_type),
        .lda = d.lda,
        .b = ptrs.ptr + d.a.len,
        .b_lens = lens.ptr + d.a.len,
        .b_count = d.b.len,
        .b_type = @intFromEnum(d.b_type),
        .ldb = d.ldb,
        .beta_re = d.beta.re,
        .beta_im = d.beta.im,
        .c = cptrs.ptr,
        .c_lens = lens.ptr + cb,
        .c_count = d.c.len,
        .c_type = @intFromEnum(d.c_type),
        .ldc = d.ldc,
        .compute_type = @intFromEnum(d.compute_type),
        .layout = if (d.layout == .row_major) c.GS_LAYOUT_ROW_MAJOR else c.GS_LAYOUT_COL_MAJOR,
        .algo = @intFromEnum(d.algo),
    };
    try check(c.gs_host_gemm_batched_ex(ctx.handle, &x));
}
