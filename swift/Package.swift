// swift-tools-version:5.9
// The C-ABI module over libtsugumi_cuda.so and the Swift shim that keeps the
// reference's MoE encoder names.  In the reference's own Package.swift the
// two targets are added beside `Tsugumi`, which then depends on
// "TsugumiCUDA"; standing alone, this manifest builds both as a library.
// TSUGUMI_CUDA_LIB is the folder that holds libtsugumi_cuda.so.
import PackageDescription
import Foundation

let libDir = ProcessInfo.processInfo.environment["TSUGUMI_CUDA_LIB"] ?? "../tsugumi_b200"

let package = Package(
    name: "TsugumiCUDA",
    products: [
        .library(name: "TsugumiCUDA", targets: ["TsugumiCUDA"]),
    ],
    targets: [
        .target(
            name: "CTsugumiCUDA",
            linkerSettings: [
                .unsafeFlags(["-L\(libDir)", "-Xlinker", "-rpath", "-Xlinker", libDir]),
            ]),
        .target(name: "TsugumiCUDA", dependencies: ["CTsugumiCUDA"]),
    ]
)
