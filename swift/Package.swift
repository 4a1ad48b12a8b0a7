// swift-tools-version:5.9
// Swift on Linux package exposing the B200 backend to YumeLayersCore callers.
// Not compiled in this repository's build: the image has no Swift toolchain.
// Point LIBYUMECUDA_DIR at the directory holding libyumecuda.so.
import PackageDescription
import Foundation

let libDir = ProcessInfo.processInfo.environment["LIBYUMECUDA_DIR"] ?? "../yumelayers_b200"

let package = Package(
    name: "YumeLayersB200",
    products: [.library(name: "YumeLayersB200", targets: ["YumeLayersB200"])],
    targets: [
        .systemLibrary(name: "YumeCUDA", path: "Sources/YumeCUDA"),
        .target(
            name: "YumeLayersB200",
            dependencies: ["YumeCUDA"],
            linkerSettings: [.unsafeFlags(["-L\(libDir)", "-Xlinker", "-rpath", "-Xlinker", libDir])]),
    ]
)
