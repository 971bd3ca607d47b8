// TsugumiCUDA.swift -- the reference's MoE encoder classes over the C ABI of
// libtsugumi_cuda.so (module CTsugumiCUDA).
//
// Names, argument labels and thrown error kinds follow
// Sources/Tsugumi/Kernels/MoE/MoE.swift and Sources/Tsugumi/Kernels/Prefill/MoE/*.swift,
// so the runners' call sites (RealForwardRunner.swift:3079-3330, :1840-2640,
// QwenForwardRunner.swift:1460-1612) change only in what they pass: a Metal
// buffer plus byte offset becomes a device address, and the command buffer
// becomes the context's CUDA stream.  Every call enqueues on that stream and
// returns at once; `CUDAContext.synchronize()` plays
// MetalContext.checkCommandBufferError.
import CTsugumiCUDA

/// A device address (the analogue of `MTLBuffer` + `byteOffset`).
public typealias DevicePointer = UnsafeMutableRawPointer

public struct CUDAStatusError: Error, CustomStringConvertible {
    public let status: tsg_status
    public let message: String
    public var description: String { "tsugumi_cuda status \(status.rawValue): \(message)" }
}

/// PrefillMoEGroupingError (PrefillMoEGrouping.swift:52-88): the library's
/// message carries the reference's text ("route token 3 is out of range", ...).
public enum PrefillMoEGroupingError: Error {
    case invalidMetadata(String)
    case invalidArgument(String)
}

/// The "declined" path of the reference's encoders (an Int 0 / Bool false
/// return there): the caller takes another path.
public struct PathDeclined: Error { public let message: String }

@inline(__always)
func check(_ st: tsg_status, _ ctx: tsg_ctx?) throws {
    if st == TSG_OK { return }
    let msg = ctx.map { String(cString: tsg_last_error_string($0)) } ?? ""
    switch st {
    case TSG_ERR_METADATA: throw PrefillMoEGroupingError.invalidMetadata(msg)
    case TSG_ERR_INVALID_ARG: throw PrefillMoEGroupingError.invalidArgument(msg)
    case TSG_ERR_UNSUPPORTED_SHAPE: throw PathDeclined(message: msg)
    default: throw CUDAStatusError(status: st, message: msg)
    }
}

/// MetalContext analogue: one device, one stream, the library's workspace.
/// Not Sendable, like the reference's kernel objects (MoE.swift:505-512).
public final class CUDAContext {
    public let handle: tsg_ctx

    /// `stream` is a `cudaStream_t`, or nil for the legacy default stream.
    public init(device: Int32, stream: UnsafeMutableRawPointer? = nil) throws {
        var h: tsg_ctx? = nil
        try check(tsg_ctx_create(device, stream, &h), nil)
        handle = h!
    }

    deinit { _ = tsg_ctx_destroy(handle) }

    public func setStream(_ stream: UnsafeMutableRawPointer?) throws {
        try check(tsg_ctx_set_stream(handle, stream), handle)
    }

    public func setOption(_ name: String, _ value: Int64) throws {
        try check(tsg_ctx_set_option(handle, name, value), handle)
    }

    /// Sizes the workspace once, so later calls allocate nothing.
    public func reserve(layer: MoELayerWeights, maxTokens: UInt32) throws {
        try check(tsg_ctx_reserve(handle, layer.handle, maxTokens), handle)
    }

    /// checkCommandBufferError (MetalContext.swift:40-45).
    public func synchronize() throws { try check(tsg_sync(handle), handle) }
}

/// One layer's resident weights (router, expert blobs in the MoEExpertOffsets
/// layout, optional shared expert and its gate row).
public final class MoELayerWeights {
    public let handle: tsg_moe_layer

    public init(context: CUDAContext, descriptor: tsg_moe_layer_desc) throws {
        var d = descriptor
        var h: tsg_moe_layer? = nil
        try check(tsg_moe_layer_create(context.handle, &d, &h), context.handle)
        handle = h!
    }

    deinit { _ = tsg_moe_layer_destroy(handle) }
}

/// MoE (MoE.swift:123-199): the decode router and routed phases of a layer.
public final class MoE {
    public let context: CUDAContext
    public let layer: MoELayerWeights

    public init(context: CUDAContext, layer: MoELayerWeights) {
        self.context = context
        self.layer = layer
    }

    /// encodeRouterGemma4BF16 / encodeRouterGemma4BF16Rows (MoE.swift:259-302, :413-466).
    public func encodeRouterGemma4BF16(hidden: UnsafeRawPointer, hiddenStride: UInt32, rows: UInt32,
                                       outIndices: UnsafeMutablePointer<UInt32>,
                                       outWeights: UnsafeMutablePointer<Float>,
                                       outWeightsF16: UnsafeMutablePointer<UInt16>? = nil) throws {
        try check(tsg_router_topk(context.handle, layer.handle, hidden, hiddenStride, rows,
                                  outIndices, outWeights, outWeightsF16), context.handle)
    }

    /// encodeRouterLogitsBF16 (MoE.swift:316-345): fp32 logits [rows][E], no select.
    public func encodeRouterLogitsBF16(hidden: UnsafeRawPointer, hiddenStride: UInt32, rows: UInt32,
                                       outLogits: UnsafeMutablePointer<Float>) throws {
        try check(tsg_router_logits(context.handle, layer.handle, hidden, hiddenStride, rows,
                                    outLogits), context.handle)
    }

    /// encodeRoutedPersistentPhase1U16Load + encodeRoutedPersistentPhase2Reduce
    /// (MoE.swift:529-644) for caller-supplied routing:
    /// y = residual + shared + sum_k w_k * expert_k(x).
    public func encodeRoutedPersistentPhases(x: UnsafeRawPointer, xStride: UInt32, rows: UInt32,
                                             indices: UnsafePointer<UInt32>,
                                             routingWeights: UnsafePointer<Float>,
                                             residual: UnsafePointer<Float>?,
                                             y: DevicePointer, yStride: UInt32,
                                             yType: tsg_dtype = TSG_DTYPE_BF16) throws {
        try check(tsg_moe_experts_decode(context.handle, layer.handle, x, xStride, rows, indices,
                                         routingWeights, residual, y, yStride, yType),
                  context.handle)
    }

    /// The whole block for a router-driven batch (the runners' per-layer
    /// sequence): router, permutation, experts, shared expert, combine.
    public func encodeBlock(hidden: UnsafeRawPointer, hiddenStride: UInt32, rows: UInt32,
                            residual: UnsafePointer<Float>?, y: DevicePointer, yStride: UInt32,
                            yType: tsg_dtype = TSG_DTYPE_BF16) throws {
        try check(tsg_moe_block_forward(context.handle, layer.handle, hidden, hiddenStride, rows,
                                        residual, y, yStride, yType), context.handle)
    }
}

/// PrefillRouter (PrefillRouter.swift:127-258).
public enum PrefillRouter {
    public static func makeTokenExpertPairs(context: CUDAContext, indices: UnsafePointer<UInt32>,
                                            weightsF16: UnsafePointer<UInt16>?, queryCount: UInt32,
                                            topK: UInt32,
                                            out: UnsafeMutablePointer<tsg_token_expert_pair>) throws {
        try check(tsg_make_token_expert_pairs(context.handle, indices, weightsF16, queryCount, topK,
                                              out), context.handle)
    }
}

/// PrefillMoEGrouping.groupTokenExpertPairs (PrefillMoEGrouping.swift:91-201),
/// on the device.  Per-pair errors surface from `CUDAContext.synchronize()`.
public enum PrefillMoEGrouping {
    public struct Outputs {
        public var sortedPairs: UnsafeMutablePointer<tsg_token_expert_pair>
        public var perExpertOffsets: UnsafeMutablePointer<UInt32>
        public var perExpertCounts: UnsafeMutablePointer<UInt32>
        public var groups: UnsafeMutablePointer<tsg_moe_group>
        public var groupCount: UnsafeMutablePointer<UInt32>
        public var tiles: UnsafeMutablePointer<tsg_moe_tile>
        public var tileCount: UnsafeMutablePointer<UInt32>
    }

    public static func groupTokenExpertPairs(context: CUDAContext,
                                             pairs: UnsafePointer<tsg_token_expert_pair>,
                                             pairCount: UInt32, queryCount: Int32, topK: Int32,
                                             numExperts: Int32, tileExpertCount: Int32 = 16,
                                             expertSortKeys: UnsafePointer<UInt64>? = nil,
                                             tileBreakAfterGroup: Int32 = -1,
                                             into o: Outputs) throws {
        try check(tsg_moe_group_pairs(context.handle, pairs, pairCount, queryCount, topK,
                                      numExperts, tileExpertCount, expertSortKeys,
                                      expertSortKeys == nil ? 0 : numExperts, tileBreakAfterGroup,
                                      o.sortedPairs, o.perExpertOffsets, o.perExpertCounts,
                                      o.groups, o.groupCount, o.tiles, o.tileCount),
                  context.handle)
    }
}

/// PrefillRoutedGEMMPlanner.plan (PrefillGroupedRoutedMoE.swift:42-83), on
/// host arrays.
public enum PrefillRoutedGEMMPlanner {
    public struct Batch {
        public var rows: UInt32
        public var blocks: ArraySlice<tsg_routed_gemm_block>
    }

    public static func plan(groups: [tsg_moe_group], maxRowsPerBatch: UInt32,
                            tileRows: UInt32 = 64) throws -> [Batch] {
        let total = groups.reduce(0) { $0 + Int($1.pair_count) }
        let cap = total + groups.count + 4
        var blocks = [tsg_routed_gemm_block](repeating: tsg_routed_gemm_block(), count: cap)
        var rows = [UInt32](repeating: 0, count: cap)
        var first = [UInt32](repeating: 0, count: cap)
        var count = [UInt32](repeating: 0, count: cap)
        var nBlocks: UInt32 = 0
        var nBatches: UInt32 = 0
        try check(tsg_plan_routed_gemm(groups, UInt32(groups.count), maxRowsPerBatch, tileRows,
                                       &blocks, UInt32(cap), &nBlocks, &rows, &first, &count,
                                       UInt32(cap), &nBatches), nil)
        return (0..<Int(nBatches)).map { i in
            Batch(rows: rows[i], blocks: blocks[Int(first[i])..<Int(first[i] + count[i])])
        }
    }
}

/// PrefillGroupedRoutedMoE.encodeStreamedTiled (PrefillGroupedRoutedMoE.swift:931-1051)
/// + PrefillMoE.encodeReduceTokenMajor for caller-supplied routing.
public final class PrefillGroupedRoutedMoE {
    public let context: CUDAContext
    public let layer: MoELayerWeights

    public init(context: CUDAContext, layer: MoELayerWeights) {
        self.context = context
        self.layer = layer
    }

    public func encodeStreamedTiled(x: UnsafeRawPointer, xStride: UInt32, rows: UInt32,
                                    indices: UnsafePointer<UInt32>, weights: UnsafePointer<Float>,
                                    residual: UnsafePointer<Float>?, y: DevicePointer,
                                    yStride: UInt32, yType: tsg_dtype = TSG_DTYPE_BF16) throws {
        try check(tsg_moe_experts_prefill(context.handle, layer.handle, x, xStride, rows, indices,
                                          weights, residual, y, yStride, yType), context.handle)
    }
}

/// PrefillMoE.encodeReduceTokenMajor (PrefillMoE.swift:11-39).
public enum PrefillMoE {
    public static func encodeReduceTokenMajor(context: CUDAContext, partials: UnsafePointer<UInt16>,
                                              weights: UnsafePointer<Float>, queryCount: UInt32,
                                              topK: UInt32, d: UInt32, h2: DevicePointer,
                                              h2Type: tsg_dtype = TSG_DTYPE_BF16) throws {
        try check(tsg_moe_reduce_token_major(context.handle, partials, weights, queryCount, topK, d,
                                             h2, h2Type), context.handle)
    }
}

/// SharedExpertRuntime.encode (SharedExpertInt4.swift:115-136) with the Qwen
/// sigmoid gate (QwenKernels.encodeMoESharedGate, QwenKernels.swift:311-355).
public final class SharedExpertRuntime {
    public let context: CUDAContext
    public let layer: MoELayerWeights

    public init(context: CUDAContext, layer: MoELayerWeights) {
        self.context = context
        self.layer = layer
    }

    public func encode(x: UnsafeRawPointer, xStride: UInt32, rows: UInt32, y: DevicePointer,
                       yStride: UInt32, yType: tsg_dtype = TSG_DTYPE_BF16) throws {
        try check(tsg_shared_expert(context.handle, layer.handle, x, xStride, rows, y, yStride,
                                    yType), context.handle)
    }
}
