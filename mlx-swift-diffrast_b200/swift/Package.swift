// swift-tools-version:5.9
// Swift wrapper over libdiffrast.so (include/diffrast.h).  Source only: it has
// not been compiled (no Swift toolchain where it was written).
import PackageDescription

let package = Package(
    name: "DiffRastB200",
    products: [.library(name: "DiffRast", targets: ["DiffRast"])],
    targets: [
        .systemLibrary(name: "CDiffRast", path: "Sources/CDiffRast"),
        .target(name: "DiffRast", dependencies: ["CDiffRast"],
                linkerSettings: [.linkedLibrary("diffrast")]),
    ]
)
