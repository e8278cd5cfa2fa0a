// Minimal declarations of the public SQLite 3 C API used by the HRM store.  The build links against the system
// runtime library (libsqlite3.so.0); no SQLite development headers are required.
#pragma once
#ifdef __cplusplus
extern "C" {
#endif

typedef struct sqlite3 sqlite3;
typedef struct sqlite3_stmt sqlite3_stmt;
typedef void (*sqlite3_destructor_type)(void*);

#define SQLITE_OK 0
#define SQLITE_ROW 100
#define SQLITE_DONE 101
#define SQLITE_OPEN_READONLY 0x00000001
#define SQLITE_OPEN_READWRITE 0x00000002
#define SQLITE_OPEN_CREATE 0x00000004
#define SQLITE_TRANSIENT ((sqlite3_destructor_type)-1)

int sqlite3_open_v2(const char* filename, sqlite3** db, int flags, const char* vfs);
int sqlite3_close(sqlite3* db);
int sqlite3_exec(sqlite3* db, const char* sql, int (*cb)(void*, int, char**, char**), void* arg, char** errmsg);
void sqlite3_free(void* p);
const char* sqlite3_errmsg(sqlite3* db);
int sqlite3_prepare_v2(sqlite3* db, const char* sql, int nbyte, sqlite3_stmt** stmt, const char** tail);
int sqlite3_step(sqlite3_stmt* stmt);
int sqlite3_reset(sqlite3_stmt* stmt);
int sqlite3_finalize(sqlite3_stmt* stmt);
int sqlite3_clear_bindings(sqlite3_stmt* stmt);
int sqlite3_bind_int(sqlite3_stmt* stmt, int idx, int v);
int sqlite3_bind_text(sqlite3_stmt* stmt, int idx, const char* v, int n, sqlite3_destructor_type d);
int sqlite3_bind_blob(sqlite3_stmt* stmt, int idx, const void* v, int n, sqlite3_destructor_type d);
int sqlite3_column_int(sqlite3_stmt* stmt, int col);
const unsigned char* sqlite3_column_text(sqlite3_stmt* stmt, int col);
const void* sqlite3_column_blob(sqlite3_stmt* stmt, int col);
int sqlite3_column_bytes(sqlite3_stmt* stmt, int col);

#ifdef __cplusplus
}
#endif
