// PagePool.swift -- the reference's paged KV cache API over libgadeonkv.so.
//
// A drop-in for leok7v/gadeon's PagePool (LLM/src/CoreML/PagedAttention.swift
// :21-287) and hostFlashDecode (:317-366): the same names, argument labels and
// error behaviour, with the pages in HBM of a B200 instead of MLMultiArrays.
// Page contents, block tables and the free list follow the library's block
// pool (see include/gadeon_kv.h); host arrays ([UInt16] fp16 bit patterns,
// [Float]) are plain Swift arrays, which the library stages through device
// memory, so callers need no CUDA code of their own.
//
// Differences a caller sees:
//   * Pages live in a GKVBlockPool (one attention layer's physical pool on one
//     GPU).  PagePool(P:kvHeads:dh:) uses the pool shared by every PagePool of
//     that geometry (GKVBlockPool.shared), sized by configureShared(...); the
//     pool's sequence is created on the first append/seed, so the
//     initializer does not throw, as the Swift's does not.
//   * kPage/vPage/tileAt return [UInt16] copies instead of MLMultiArrays.
//   * pagedFlashBatched takes no ANE tile program: the library's tensor-core
//     chunk kernel computes every row.
import CGadeonKV

/// A failing C ABI call: its gkv_status and gkv_last_error() message.
public struct GKVError: Error, CustomStringConvertible {
    public let code: Int32
    public let message: String
    public var description: String { "gkv error \(code): \(message)" }
}

@inline(__always) func gkvTry(_ rc: Int32) throws {
    if rc != 0 { throw GKVError(code: rc, message: String(cString: gkv_last_error())) }
}

/// The page store of one full-attention layer on one GPU (gkv_pool): the
/// physical K/V pages, the free list and every sequence's block table.
public final class GKVBlockPool {
    public let handle: OpaquePointer
    public let P: Int, kvHeads: Int, dh: Int

    public init(device: Int32 = 0, P: Int, kvHeads: Int, dh: Int, pages: Int, maxSeqs: Int,
                maxPagesPerSeq: Int, seed: UInt64 = 0) throws {
        var cfg = gkv_pool_config(device: device, kv_heads: Int32(kvHeads), head_dim: Int32(dh),
                                  page_tokens: Int32(P), num_pages: Int32(pages), max_seqs: Int32(maxSeqs),
                                  max_pages_per_seq: Int32(maxPagesPerSeq), seed: seed)
        var h: OpaquePointer?
        try gkvTry(gkv_pool_create(&cfg, &h))
        handle = h!
        self.P = P
        self.kvHeads = kvHeads
        self.dh = dh
    }

    deinit { gkv_pool_destroy(handle) }

    public var freePageCount: Int {
        var n: Int32 = 0
        _ = gkv_free_page_count(handle, &n)
        return Int(n)
    }

    // ---- the pool shared by PagePool(P:kvHeads:dh:)
    public struct SharedSize {
        public var device: Int32 = 0
        public var pages = 65536
        public var maxSeqs = 1024
        public var maxPagesPerSeq = 16384
        public init() {}
    }
    private static var sharedSize = SharedSize()
    private static var sharedPools: [String: GKVBlockPool] = [:]

    /// Sets the size of the pools created by shared(P:kvHeads:dh:) from now on.
    public static func configureShared(_ size: SharedSize) { sharedSize = size }

    /// The pool every PagePool(P:kvHeads:dh:) of this geometry uses.
    public static func shared(P: Int, kvHeads: Int, dh: Int) throws -> GKVBlockPool {
        let key = "\(P)x\(kvHeads)x\(dh)"
        if let p = sharedPools[key] { return p }
        let s = sharedSize
        let p = try GKVBlockPool(device: s.device, P: P, kvHeads: kvHeads, dh: dh, pages: s.pages,
                                 maxSeqs: s.maxSeqs, maxPagesPerSeq: s.maxPagesPerSeq)
        sharedPools[key] = p
        return p
    }
}

/// One sequence's K/V cache: the reference's PagePool (PagedAttention.swift:21).
public final class PagePool {
    public let P: Int
    public let kvHeads: Int
    public let dh: Int
    private let explicitPool: GKVBlockPool?
    private var pool: GKVBlockPool?
    private var seq: Int32 = -1

    /// init(P:kvHeads:dh:) (:40): a new, empty cache in the shared pool of
    /// this geometry.
    public init(P: Int, kvHeads: Int, dh: Int) {
        self.P = P
        self.kvHeads = kvHeads
        self.dh = dh
        explicitPool = nil
    }

    /// A new, empty cache in a given block pool.
    public init(pool: GKVBlockPool) {
        P = pool.P
        kvHeads = pool.kvHeads
        dh = pool.dh
        explicitPool = pool
    }

    private init(pool: GKVBlockPool, seq: Int32) {
        P = pool.P
        kvHeads = pool.kvHeads
        dh = pool.dh
        explicitPool = pool
        self.pool = pool
        self.seq = seq
    }

    deinit {
        if let p = pool, seq >= 0 { _ = gkv_seq_release(p.handle, seq) }
    }

    /// The pool and sequence, made on first use.
    private func bound() throws -> (GKVBlockPool, Int32) {
        if let p = pool { return (p, seq) }
        let p = try explicitPool ?? GKVBlockPool.shared(P: P, kvHeads: kvHeads, dh: dh)
        var id: Int32 = -1
        try gkvTry(gkv_seq_create(p.handle, &id))
        pool = p
        seq = id
        return (p, id)
    }

    /// length (:27): positions written.
    public var length: Int {
        guard let p = pool else { return 0 }
        var n: Int64 = 0
        _ = gkv_seq_length(p.handle, seq, &n)
        return Int(n)
    }

    /// pageCount (:79).
    public var pageCount: Int {
        guard let p = pool else { return 0 }
        var n: Int32 = 0
        _ = gkv_seq_page_count(p.handle, seq, &n)
        return Int(n)
    }

    /// append(k:v:) (:85-94): one position, k and v [kvHeads, dh] fp16.
    public func append(k: [UInt16], v: [UInt16]) throws {
        precondition(k.count == kvHeads * dh && v.count == kvHeads * dh, "append: k/v must hold kvHeads*dh values")
        let (p, id) = try bound()
        var ids = id
        var one: Int32 = 1
        try k.withUnsafeBytes { kb in
            try v.withUnsafeBytes { vb in
                try gkvTry(gkv_append(p.handle, 1, &ids, &one, kb.baseAddress, vb.baseAddress, nil))
            }
        }
    }

    /// append(k:v:) with device (or page-locked) buffers on a CUDA stream.
    public func append(k: UnsafeRawPointer, v: UnsafeRawPointer, stream: UnsafeMutableRawPointer?) throws {
        let (p, id) = try bound()
        var ids = id
        var one: Int32 = 1
        try gkvTry(gkv_append(p.handle, 1, &ids, &one, k, v, stream))
    }

    /// seed(K:V:count:) (:99-112): an empty cache from [kvHeads, count, dh] fp16.
    public func seed(K: [UInt16], V: [UInt16], count: Int) throws {
        precondition(K.count >= kvHeads * count * dh && V.count >= kvHeads * count * dh, "seed: K/V too short")
        let (p, id) = try bound()
        try K.withUnsafeBytes { kb in
            try V.withUnsafeBytes { vb in
                try gkvTry(gkv_seed(p.handle, id, kb.baseAddress, vb.baseAddress, Int64(count), nil))
            }
        }
    }

    /// tileAt(_:_:_:) (:151-161): positions [start, start + count) as
    /// [kvHeads, tileP, dh] fp16 K and V, rows count..tileP-1 zero.
    public func tileAt(_ start: Int, _ count: Int, _ tileP: Int) throws -> ([UInt16], [UInt16]) {
        let (p, id) = try bound()
        var k = [UInt16](repeating: 0, count: kvHeads * tileP * dh)
        var v = [UInt16](repeating: 0, count: kvHeads * tileP * dh)
        try k.withUnsafeMutableBytes { kb in
            try v.withUnsafeMutableBytes { vb in
                try gkvTry(gkv_tile_at(p.handle, id, Int64(start), Int64(count), Int32(tileP), kb.baseAddress,
                                       vb.baseAddress, nil))
            }
        }
        return (k, v)
    }

    /// truncate(to:) (:181-189): whole pages past the new length return to
    /// the free list (last first); the kept tail keeps its stale rows.
    public func truncate(to newLength: Int) {
        guard let p = pool else {
            precondition(newLength == 0, "truncate past the end")
            return
        }
        var id = seq
        var n = Int64(newLength)
        precondition(gkv_truncate(p.handle, 1, &id, &n) == 0, String(cString: gkv_last_error()))
    }

    /// clone() (:199-210): shares every full page, copies a partial tail.
    public func clone() throws -> PagePool {
        let (p, id) = try bound()
        var dst: Int32 = -1
        try gkvTry(gkv_clone_seq(p.handle, id, &dst, nil))
        return PagePool(pool: p, seq: dst)
    }

    /// compact() (:225-252): K and V as [kvHeads, length, dh] fp16.
    public func compact() -> (k: [UInt16], v: [UInt16]) {
        let n = kvHeads * length * dh
        var k = [UInt16](repeating: 0, count: n)
        var v = [UInt16](repeating: 0, count: n)
        guard let p = pool, n > 0 else { return (k, v) }
        k.withUnsafeMutableBytes { kb in
            v.withUnsafeMutableBytes { vb in
                precondition(gkv_compact_seq(p.handle, seq, kb.baseAddress, vb.baseAddress, nil) == 0,
                             String(cString: gkv_last_error()))
            }
        }
        return (k, v)
    }

    /// fromCompact(k:v:length:P:kvHeads:dh:) (:256-264).
    public static func fromCompact(k: [UInt16], v: [UInt16], length: Int, P: Int, kvHeads: Int,
                                   dh: Int) throws -> PagePool {
        let pool = PagePool(P: P, kvHeads: kvHeads, dh: dh)
        if length > 0 { try pool.seed(K: k, V: v, count: length) }
        return pool
    }

    /// kPage(_:) / vPage(_:) (:80-81): page i as stored, [kvHeads, P, dh] fp16.
    public func kPage(_ i: Int) -> [UInt16] { page(i).0 }
    public func vPage(_ i: Int) -> [UInt16] { page(i).1 }

    private func page(_ i: Int) -> ([UInt16], [UInt16]) {
        guard let p = pool else { preconditionFailure("page \(i) of an empty cache") }
        var table = [Int32](repeating: 0, count: pageCount)
        var n: Int32 = 0
        precondition(gkv_export_table(p.handle, seq, &table, Int32(table.count), &n) == 0 && i < Int(n),
                     "page \(i) of a cache with \(n) pages")
        var k = [UInt16](repeating: 0, count: kvHeads * P * dh)
        var v = [UInt16](repeating: 0, count: kvHeads * P * dh)
        precondition(gkv_export_page(p.handle, table[i], &k, &v) == 0, String(cString: gkv_last_error()))
        return (k, v)
    }

    /// floats32() (:46-62): per kv head, the positions [0, length) widened to
    /// fp32 ([length * dh] each).
    public func floats32() -> (k: [[Float]], v: [[Float]]) {
        let (k, v) = compact()
        let per = length * dh
        var kf = [[Float]](), vf = [[Float]]()
        for h in 0 ..< kvHeads {
            kf.append(k[h * per ..< (h + 1) * per].map { Float(Float16(bitPattern: $0)) })
            vf.append(v[h * per ..< (h + 1) * per].map { Float(Float16(bitPattern: $0)) })
        }
        return (kf, vf)
    }

    fileprivate var ids: (OpaquePointer, Int32)? {
        guard let p = pool else { return nil }
        return (p.handle, seq)
    }
}

/// hostFlashDecode(q:pool:G:) (PagedAttention.swift:317-366): the newest
/// query q [kvHeads, G, dh] fp16 over every one of the pool's length keys,
/// scale dh^-0.5; returns [kvHeads*G*dh] fp32.  An empty pool gives zeros.
public func hostFlashDecode(q: [UInt16], pool: PagePool, G: Int) -> [Float] {
    var out = [Float](repeating: 0, count: pool.kvHeads * G * pool.dh)
    guard let bound = pool.ids, pool.length > 0 else { return out }
    let (h, id) = bound
    precondition(q.count == pool.kvHeads * G * pool.dh, "hostFlashDecode: q must hold kvHeads*G*dh values")
    var seq = id
    let scale = Float(1.0 / Double(pool.dh).squareRoot())
    q.withUnsafeBytes { qb in
        out.withUnsafeMutableBufferPointer { ob in
            precondition(gkv_attend(h, 1, &seq, 1, Int32(G), qb.baseAddress, ob.baseAddress, scale, nil) == 0,
                         String(cString: gkv_last_error()))
        }
    }
    return out
}

/// pagedFlashBatched(q:pool:tile:s0GlobalPos:sCount:G:) (PagedAttention.swift
/// :376-416) without the tile program: query rows q [kvHeads, sCount, G, dh]
/// fp16 at global positions s0GlobalPos + s, each seeing keys
/// [0, s0GlobalPos + s]; returns the normalized [kvHeads, sCount, G, dh]
/// fp32 result.  The rows must be the pool's last sCount positions (append
/// the chunk first, as Engine.batchedAttn does).  pF16: the softmax weights
/// rounded once to fp16 on the tensor-core path (GKV_ATTEND_P_F16), as the
/// Metal attn_batch_mm computes them (Kernels.metal:1891-1912).
public func pagedFlashBatched(q: [UInt16], pool: PagePool, s0GlobalPos: Int, sCount: Int,
                              G: Int, pF16: Bool = false) throws -> [Float] {
    guard let bound = pool.ids, s0GlobalPos + sCount == pool.length else {
        throw GKVError(code: 1, message: "rows must be the pool's last \(sCount) positions")
    }
    let (h, id) = bound
    var out = [Float](repeating: 0, count: pool.kvHeads * sCount * G * pool.dh)
    var seq = id
    let scale = Float(1.0 / Double(pool.dh).squareRoot())
    let flags = UInt32(GKV_ATTEND_HEAD_MAJOR.rawValue | (pF16 ? GKV_ATTEND_P_F16.rawValue : 0))
    try q.withUnsafeBytes { qb in
        try out.withUnsafeMutableBytes { ob in
            try gkvTry(gkv_attend_ex(h, 1, &seq, Int32(sCount), Int32(G), qb.baseAddress, ob.baseAddress, scale,
                                     flags, nil))
        }
    }
    return out
}

/// Engine.verifyAttn (LLM/src/CoreML/Engine.swift:2620-2646) in one call:
/// appends the L rows k, v [kvHeads, L, dh] fp16 and attends query row s of
/// q [kvHeads, L, G, dh] over the pool so far (causal among the rows);
/// returns attn_out [kvHeads, L, G, dh] fp16.
public func verifyAttn(pool: PagePool, k: [UInt16], v: [UInt16], q: [UInt16], L: Int, G: Int) throws -> [UInt16] {
    if pool.ids == nil { try pool.seed(K: [], V: [], count: 0) }
    guard let bound = pool.ids else { throw GKVError(code: 1, message: "no cache") }
    let (h, id) = bound
    var out = [UInt16](repeating: 0, count: pool.kvHeads * L * G * pool.dh)
    var seq = id
    let scale = Float(1.0 / Double(pool.dh).squareRoot())
    let flags = UInt32(GKV_ATTEND_HEAD_MAJOR.rawValue | GKV_ATTEND_OUT_F16.rawValue)
    try k.withUnsafeBytes { kb in
        try v.withUnsafeBytes { vb in
            try q.withUnsafeBytes { qb in
                try out.withUnsafeMutableBytes { ob in
                    try gkvTry(gkv_append_attend_ex(h, 1, &seq, Int32(L), Int32(G), kb.baseAddress, vb.baseAddress,
                                                    qb.baseAddress, ob.baseAddress, scale, flags, nil))
                }
            }
        }
    }
    return out
}
