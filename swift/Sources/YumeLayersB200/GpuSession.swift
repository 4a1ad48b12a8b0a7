// Swift mirror of the reference's GPU runtime types over the B200 backend's
// C ABI (include/yume_c.h).  It keeps the names, argument meaning and the
// functional style (every op returns a new tensor) of
//   GpuSession   -- Sources/YumeLayersCore/GpuTraining.swift:4-151 and the
//                   ops of GpuSessionOps.swift / GpuSessionNormGrad.swift,
//   GPUTensor    -- Sources/YumeLayersCore/GPUTensor.swift:9-143,
// so that the reference's layers can switch backends by changing imports.
//
// Not compiled in this repository's build: the image has no Swift toolchain.
// The Python mirror (yumelayers_b200/session.py) exercises the same entry
// points in the tests.
//
// Differences that follow from the backend, not from the API:
//   * a GPU that does not finish within the deadline makes end()/wait()
//     throw YumeCUDAError(YL_ERR_TIMEOUT) instead of calling exit(70)
//     (GpuTraining.swift:92-97);
//   * tensors are owned by the device's stream-ordered pool, so release in
//     deinit is safe while queued work still reads them.
import Foundation
import YumeCUDA

public struct YumeCUDAError: Error, CustomStringConvertible {
    public let status: yl_status
    public let message: String
    public var description: String { "yl_status \(status.rawValue): \(message)" }
}

/// Throws for a non-OK status; a shape error stops the program the way the
/// reference's preconditions do (GpuSessionOps.swift:112, 122, ...).
@inline(__always)
func check(_ s: yl_status) throws {
    guard s == YL_OK else {
        let msg = String(cString: yl_last_error_message())
        precondition(s != YL_ERR_SHAPE, msg)
        throw YumeCUDAError(status: s, message: msg)
    }
}

/// One GPU and its stream (the role of MetalEngine, MetalEngine.swift:6-60).
public final class Engine {
    let ctx: OpaquePointer

    public init(device: Int32 = 0) throws {
        var c: OpaquePointer?
        try check(yl_ctx_create(device, &c))
        ctx = c!
    }

    deinit { _ = yl_ctx_destroy(ctx) }
}

/// rows x cols fp32 tensor in device memory (GPUTensor.swift:9-143).
public final class GPUTensor {
    let engine: Engine
    let handle: OpaquePointer
    public let rows: Int
    public let cols: Int
    public var n: Int { rows * cols }

    public init(engine: Engine, rows: Int, cols: Int) throws {
        var t: OpaquePointer?
        try check(yl_tensor_create(engine.ctx, Int32(rows), Int32(cols), nil, &t))
        self.engine = engine
        self.handle = t!
        self.rows = rows
        self.cols = cols
    }

    public init(engine: Engine, data: [Float], rows: Int) throws {
        precondition(rows > 0 && data.count % rows == 0,
                     "GPUTensor: rows=\(rows) must divide \(data.count) elements")
        var t: OpaquePointer?
        try data.withUnsafeBufferPointer {
            try check(yl_tensor_create(engine.ctx, Int32(rows), Int32(data.count / rows),
                                       $0.baseAddress, &t))
        }
        self.engine = engine
        self.handle = t!
        self.rows = rows
        self.cols = data.count / rows
    }

    deinit { _ = yl_tensor_release(handle) }

    var ptr: UnsafeMutablePointer<Float> { yl_tensor_data(handle)! }

    public func toArray() throws -> [Float] {
        var out = [Float](repeating: 0, count: n)
        try out.withUnsafeMutableBufferPointer {
            try check(yl_tensor_download(handle, $0.baseAddress, n))
        }
        return out
    }

    public func setData(_ data: [Float]) throws {
        precondition(data.count == n)
        try data.withUnsafeBufferPointer { try check(yl_tensor_upload(handle, $0.baseAddress, n)) }
    }

    public func copyFrom(_ src: GPUTensor) throws {
        precondition(src.n == n)
        try check(yl_copy(engine.ctx, ptr, src.ptr, n))
    }

    public func setValue(_ index: Int, _ value: Float) throws {
        precondition(index >= 0 && index < n, "setValue: index \(index) outside \(n)")
        try check(yl_tensor_set_value(handle, index, value))
    }

    public func getValue(_ index: Int) throws -> Float {
        precondition(index >= 0 && index < n, "getValue: index \(index) outside \(n)")
        var v: Float = 0
        try check(yl_tensor_get_value(handle, index, &v))
        return v
    }
}

/// Work recorded between begin() and end()/commit() (GpuTraining.swift:4-151).
public final class GpuSession {
    public let engine: Engine
    /// The reference's hang bound (GpuTraining.swift:30), in seconds.
    public static var gpuDeadlineSeconds: Double = 30

    public init(_ engine: Engine) { self.engine = engine }

    var ctx: OpaquePointer { engine.ctx }

    public func begin() throws { try check(yl_session_begin(ctx)) }

    /// commit() without waiting; wait() returns the device time in ms,
    /// bounded by the wall time (boundedGpuMs, GpuWaitPolicy.swift:75-87).
    public final class CommittedStep {
        let session: GpuSession
        init(_ s: GpuSession) { session = s }
        public func wait() throws -> Double {
            var ms = 0.0
            try check(yl_session_end(session.ctx, GpuSession.gpuDeadlineSeconds, &ms))
            return ms
        }
    }

    public func commit() throws -> CommittedStep {
        try check(yl_session_commit(ctx))
        return CommittedStep(self)
    }

    @discardableResult
    public func end() throws -> Double { try commit().wait() }

    func out(_ rows: Int, _ cols: Int) throws -> GPUTensor {
        try GPUTensor(engine: engine, rows: rows, cols: cols)
    }

    // ------------------------------------------------ GpuSessionOps (reference semantics)
    public func matmul(_ a: GPUTensor, _ b: GPUTensor, transA: Bool = false,
                       transB: Bool = false, M: Int, N: Int, K: Int) throws -> GPUTensor {
        let c = try out(M, N)
        try check(yl_matmul(ctx, a.ptr, b.ptr, c.ptr, Int32(M), Int32(N), Int32(K),
                            transA ? 1 : 0, transB ? 1 : 0))
        return c
    }

    public func im2col(_ x: GPUTensor, ic: Int, ih: Int, iw: Int, kh: Int, kw: Int,
                       stride: Int, pad: Int) throws -> GPUTensor {
        let oh = (ih + 2 * pad - kh) / stride + 1, ow = (iw + 2 * pad - kw) / stride + 1
        let cols = try out(ic * kh * kw, oh * ow)
        try check(yl_im2col(ctx, x.ptr, cols.ptr, Int32(ic), Int32(ih), Int32(iw), Int32(kh),
                            Int32(kw), Int32(stride), Int32(pad)))
        return cols
    }

    public func col2im(_ cols: GPUTensor, ic: Int, ih: Int, iw: Int, kh: Int, kw: Int,
                       stride: Int, pad: Int, oh: Int, ow: Int) throws -> GPUTensor {
        let g = try out(ic, ih * iw)
        try check(yl_col2im(ctx, cols.ptr, g.ptr, Int32(ic), Int32(ih), Int32(iw), Int32(kh),
                            Int32(kw), Int32(stride), Int32(pad), Int32(oh), Int32(ow)))
        return g
    }

    public func gradW(_ a: GPUTensor, _ b: GPUTensor, oc: Int, kk: Int) throws -> GPUTensor {
        let k = a.n / oc
        let c = try out(oc, kk)
        try check(yl_grad_w(ctx, a.ptr, b.ptr, c.ptr, Int32(oc), Int32(kk), Int32(k)))
        return c
    }

    public func convBackInputS1(_ dOut: GPUTensor, _ w: GPUTensor, ic: Int, oc: Int, ih: Int,
                                iw: Int, k: Int, pad: Int) throws -> GPUTensor {
        let dx = try out(ic, ih * iw)
        try check(yl_conv_back_input_s1(ctx, dOut.ptr, w.ptr, dx.ptr, Int32(ic), Int32(oc),
                                        Int32(ih), Int32(iw), Int32(k), Int32(pad)))
        return dx
    }

    public func biasRow(_ a: GPUTensor, _ b: GPUTensor) throws -> GPUTensor {
        let c = try out(a.rows, a.cols)
        try check(yl_bias_row(ctx, a.ptr, b.ptr, c.ptr, Int32(a.rows), Int32(a.cols)))
        return c
    }

    public func biasRowGrad(_ g: GPUTensor) throws -> GPUTensor {
        let o = try out(g.rows, 1)
        try check(yl_bias_row_grad(ctx, g.ptr, o.ptr, Int32(g.rows), Int32(g.cols)))
        return o
    }

    public func addBias(_ a: GPUTensor, _ bias: GPUTensor) throws -> GPUTensor {
        let c = try out(a.rows, a.cols)
        try check(yl_add_bias(ctx, a.ptr, bias.ptr, c.ptr, Int32(a.rows), Int32(a.cols)))
        return c
    }

    public func sumCols(_ a: GPUTensor) throws -> GPUTensor {
        let c = try out(1, a.cols)
        try check(yl_sum_cols(ctx, a.ptr, c.ptr, Int32(a.rows), Int32(a.cols)))
        return c
    }

    public func groupNorm(_ a: GPUTensor, groups: Int) throws -> GPUTensor {
        let c = try out(a.rows, a.cols)
        try check(yl_group_norm(ctx, a.ptr, c.ptr, Int32(a.rows), Int32(a.cols), Int32(groups)))
        return c
    }

    public func encodeGroupNormGrad(x: GPUTensor, dy: GPUTensor, groups: Int) throws -> GPUTensor {
        let c = try out(x.rows, x.cols)
        try check(yl_group_norm_grad(ctx, x.ptr, dy.ptr, c.ptr, Int32(x.rows), Int32(x.cols),
                                     Int32(groups)))
        return c
    }

    func unary(_ op: yl_unary_op, _ a: GPUTensor) throws -> GPUTensor {
        let c = try out(a.rows, a.cols)
        try check(yl_unary(ctx, Int32(op.rawValue), a.ptr, c.ptr, a.n))
        return c
    }

    func binary(_ op: yl_binary_op, _ a: GPUTensor, _ b: GPUTensor) throws -> GPUTensor {
        precondition(a.n == b.n, "binary op: \(a.n) vs \(b.n) elements")
        let c = try out(a.rows, a.cols)
        try check(yl_binary(ctx, Int32(op.rawValue), a.ptr, b.ptr, c.ptr, a.n))
        return c
    }

    public func relu(_ a: GPUTensor) throws -> GPUTensor { try unary(YL_RELU, a) }
    public func sigmoid(_ a: GPUTensor) throws -> GPUTensor { try unary(YL_SIGMOID, a) }
    public func tanh(_ a: GPUTensor) throws -> GPUTensor { try unary(YL_TANH, a) }
    public func exp(_ a: GPUTensor) throws -> GPUTensor { try unary(YL_EXP, a) }
    public func expHalf(_ a: GPUTensor) throws -> GPUTensor { try unary(YL_EXP_HALF, a) }
    public func add(_ a: GPUTensor, _ b: GPUTensor) throws -> GPUTensor { try binary(YL_ADD, a, b) }
    public func sub(_ a: GPUTensor, _ b: GPUTensor) throws -> GPUTensor { try binary(YL_SUB, a, b) }
    public func mul(_ a: GPUTensor, _ b: GPUTensor) throws -> GPUTensor { try binary(YL_MUL, a, b) }
    public func reluGrad(_ x: GPUTensor, _ dy: GPUTensor) throws -> GPUTensor {
        try binary(YL_RELU_GRAD, x, dy)
    }

    public func smul(_ a: GPUTensor, _ s: Float) throws -> GPUTensor {
        let c = try out(a.rows, a.cols)
        try check(yl_smul(ctx, s, a.ptr, c.ptr, a.n))
        return c
    }

    public func addInPlace(_ a: GPUTensor, _ b: GPUTensor) throws {
        precondition(a.n == b.n)
        try check(yl_add_in_place(ctx, a.ptr, b.ptr, a.n))
    }

    public func upsample2x(_ x: GPUTensor, c: Int, h: Int, w: Int) throws -> GPUTensor {
        let y = try out(c, 4 * h * w)
        try check(yl_upsample2x(ctx, x.ptr, y.ptr, Int32(c), Int32(h), Int32(w)))
        return y
    }

    public func downsample2x(_ x: GPUTensor, c: Int, h: Int, w: Int) throws -> GPUTensor {
        let y = try out(c, h * w)
        try check(yl_downsample2x(ctx, x.ptr, y.ptr, Int32(c), Int32(h), Int32(w)))
        return y
    }

    public func randn(seed: UInt32, rows: Int, cols: Int) throws -> GPUTensor {
        let y = try out(rows, cols)
        try check(yl_randn(ctx, y.ptr, seed, rows * cols))
        return y
    }

    public func adamUpdate(param: GPUTensor, grad: GPUTensor, m: GPUTensor, v: GPUTensor,
                           t: Int, lr: Float) throws {
        try check(yl_adam_update(ctx, param.ptr, grad.ptr, m.ptr, v.ptr, param.n, Int32(t), lr))
    }

    // ------------------------------------------------ batched B200 operators
    /// ConvLayerGPU.forward (ConvGPU.swift:57-64) over a whole NCHW batch:
    /// one implicit-GEMM launch instead of im2col + matmul + biasRow per image.
    public func conv2dForward(_ x: GPUTensor, _ w: GPUTensor, _ b: GPUTensor?, n: Int, c: Int,
                              h: Int, w width: Int, oc: Int, k: Int = 3, stride: Int = 1,
                              pad: Int = 1, residual: GPUTensor? = nil) throws -> GPUTensor {
        var d = yl_conv_desc(n: Int32(n), c: Int32(c), h: Int32(h), w: Int32(width),
                             oc: Int32(oc), k: Int32(k), stride: Int32(stride), pad: Int32(pad),
                             up: 0, up_h: 0, up_w: 0, layout: Int32(YL_LAYOUT_NCHW.rawValue))
        var oh: Int32 = 0, ow: Int32 = 0
        try check(yl_conv2d_out_shape(&d, &oh, &ow))
        let y = try out(n * oc, Int(oh) * Int(ow))
        try check(yl_conv2d_fwd(ctx, &d, x.ptr, w.ptr, b?.ptr, residual?.ptr, y.ptr))
        return y
    }

    /// GroupNorm(groups, eps) with affine gamma/beta followed by SiLU.
    public func groupNormSiLU(_ x: GPUTensor, n: Int, c: Int, h: Int, w: Int, groups: Int = 32,
                              eps: Float = 1e-6, gamma: GPUTensor?, beta: GPUTensor?)
        throws -> (y: GPUTensor, mean: GPUTensor, rstd: GPUTensor) {
        let y = try out(x.rows, x.cols)
        let mean = try out(n, groups), rstd = try out(n, groups)
        try check(yl_groupnorm_silu_fwd(ctx, x.ptr, Int32(n), Int32(c), Int32(h), Int32(w),
                                        Int32(YL_LAYOUT_NCHW.rawValue), Int32(groups), eps, 0,
                                        gamma?.ptr, beta?.ptr, 1, y.ptr, mean.ptr, rstd.ptr))
        return (y, mean, rstd)
    }
}

/// The whole joint VAE + motion-net training step (TrainContext.runStep,
/// TrainConvVAE.swift:327-362, plus the motion step, MotionTrainer.swift:
/// 450-485) on one GPU, or one rank of a data-parallel group.
public final class JointTrainer {
    let handle: OpaquePointer
    public let engine: Engine

    public init(engine: Engine, config: yl_trainer_config, comm: OpaquePointer? = nil) throws {
        var cfg = config
        var t: OpaquePointer?
        try check(yl_trainer_create(engine.ctx, &cfg, comm, &t))
        self.engine = engine
        self.handle = t!
    }

    deinit { _ = yl_trainer_destroy(handle) }

    /// frames: [3][batch][3][H][W] (frame 0, frame 16, frame k); t: [batch].
    /// Returns (VAE loss, motion loss).
    public func step(frames: [Float], t: [Float]) throws -> (Float, Float) {
        var losses = [Float](repeating: 0, count: 2)
        try frames.withUnsafeBufferPointer { f in
            try t.withUnsafeBufferPointer { tt in
                try losses.withUnsafeMutableBufferPointer { l in
                    try check(yl_trainer_step_host(handle, f.baseAddress, tt.baseAddress,
                                                   l.baseAddress))
                }
            }
        }
        return (losses[0], losses[1])
    }
}
