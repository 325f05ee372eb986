// swift-tools-version:5.9
// GadeonKV: the reference's PagePool / hostFlashDecode surface
// (leok7v/gadeon LLM/src/CoreML/PagedAttention.swift:21-366) over the C ABI
// of libgadeonkv.so (include/gadeon_kv.h).  Build with the library on the
// linker's path, e.g.
//   swift build -Xlinker -L/path/to/gadeon_b200 -Xlinker -rpath -Xlinker /path/to/gadeon_b200
import PackageDescription

let package = Package(
    name: "GadeonKV",
    products: [.library(name: "GadeonKV", targets: ["GadeonKV"])],
    targets: [
        // the C ABI as a Swift module (module.modulemap links -lgadeonkv)
        .systemLibrary(name: "CGadeonKV", path: "Sources/CGadeonKV"),
        .target(name: "GadeonKV", dependencies: ["CGadeonKV"], path: "Sources/GadeonKV"),
    ]
)
