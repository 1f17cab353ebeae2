/* The package builds against the repository's public header. */
#include "../../../../../include/diffrast.h"
