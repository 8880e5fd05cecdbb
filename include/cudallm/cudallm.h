/* Same include path as wasiqnauman/cudallm (include/cudallm/cudallm.h), so C/C++ callers that write
 * #include "cudallm/cudallm.h" build against this library unchanged. */
#include "../cudallm.h"
