// SQLite snippet store.  Schema (same as the reference store, sqlite_store.cpp:23-39 there):
//   snips(sid TEXT PRIMARY KEY, cid INTEGER, sidx INTEGER, txt TEXT, q BLOB)  +  index on cid
// journal_mode=WAL, synchronous=FULL, INSERT OR REPLACE.
#include "hrm/hrm.h"
#include "hrm/sqlite_min.h"

#include <stdexcept>

namespace hrm {
namespace {

void exec(sqlite3* db, const char* sql) {
  char* err = nullptr;
  if (sqlite3_exec(db, sql, nullptr, nullptr, &err) != SQLITE_OK) {
    std::string e = err ? err : "?";
    sqlite3_free(err);
    throw std::runtime_error(std::string("sqlite: ") + sql + ": " + e);
  }
}

Snip row(sqlite3_stmt* st) {
  Snip s;
  const unsigned char* sid = sqlite3_column_text(st, 0);
  s.sid = sid ? reinterpret_cast<const char*>(sid) : "";
  s.cid = (uint32_t)sqlite3_column_int(st, 1);
  s.sidx = (uint32_t)sqlite3_column_int(st, 2);
  const unsigned char* txt = sqlite3_column_text(st, 3);
  s.txt = txt ? reinterpret_cast<const char*>(txt) : "";
  const auto* b = static_cast<const uint8_t*>(sqlite3_column_blob(st, 4));
  s.blob.assign(b, b + sqlite3_column_bytes(st, 4));
  return s;
}

}  // namespace

Store::~Store() { close(); }

void Store::open(const std::string& path, bool writable) {
  close();
  const int flags = writable ? (SQLITE_OPEN_READWRITE | SQLITE_OPEN_CREATE) : SQLITE_OPEN_READWRITE;
  if (sqlite3_open_v2(path.c_str(), &db_, flags, nullptr) != SQLITE_OK) {
    std::string e = db_ ? sqlite3_errmsg(db_) : "?";
    close();
    throw std::runtime_error("sqlite open failed: " + path + ": " + e);
  }
  sqlite3_exec(db_, "PRAGMA journal_mode=WAL;", nullptr, nullptr, nullptr);
  sqlite3_exec(db_, "PRAGMA synchronous=FULL;", nullptr, nullptr, nullptr);
}

void Store::close() {
  if (ins_) sqlite3_finalize(ins_);
  ins_ = nullptr;
  if (db_) sqlite3_close(db_);
  db_ = nullptr;
}

void Store::create_schema() {
  exec(db_, "CREATE TABLE IF NOT EXISTS snips (sid TEXT PRIMARY KEY, cid INTEGER, sidx INTEGER, txt TEXT, q BLOB);");
  exec(db_, "CREATE INDEX IF NOT EXISTS idx_snips_cid ON snips(cid);");
}

void Store::begin() { exec(db_, "BEGIN IMMEDIATE;"); }
void Store::commit() { exec(db_, "COMMIT;"); }

void Store::put(const Snip& s) {
  if (!ins_ && sqlite3_prepare_v2(db_, "INSERT OR REPLACE INTO snips(sid,cid,sidx,txt,q) VALUES(?,?,?,?,?);", -1,
                                  &ins_, nullptr) != SQLITE_OK)
    throw std::runtime_error("sqlite prepare insert failed");
  sqlite3_reset(ins_);
  sqlite3_clear_bindings(ins_);
  sqlite3_bind_text(ins_, 1, s.sid.c_str(), -1, SQLITE_TRANSIENT);
  sqlite3_bind_int(ins_, 2, (int)s.cid);
  sqlite3_bind_int(ins_, 3, (int)s.sidx);
  sqlite3_bind_text(ins_, 4, s.txt.c_str(), -1, SQLITE_TRANSIENT);
  sqlite3_bind_blob(ins_, 5, s.blob.data(), (int)s.blob.size(), SQLITE_TRANSIENT);
  if (sqlite3_step(ins_) != SQLITE_DONE) throw std::runtime_error("sqlite insert failed");
}

static std::vector<Snip> run_select(sqlite3* db, const char* sql, int bind_cid, bool bind) {
  sqlite3_stmt* st = nullptr;
  if (sqlite3_prepare_v2(db, sql, -1, &st, nullptr) != SQLITE_OK) throw std::runtime_error("sqlite prepare failed");
  if (bind) sqlite3_bind_int(st, 1, bind_cid);
  std::vector<Snip> out;
  for (;;) {
    const int rc = sqlite3_step(st);
    if (rc == SQLITE_DONE) break;
    if (rc != SQLITE_ROW) {
      sqlite3_finalize(st);
      throw std::runtime_error("sqlite step failed");
    }
    out.push_back(row(st));
  }
  sqlite3_finalize(st);
  return out;
}

std::vector<Snip> Store::by_cid(uint32_t cid) const {
  return run_select(db_, "SELECT sid,cid,sidx,txt,q FROM snips WHERE cid=? ORDER BY sidx ASC;", (int)cid, true);
}

std::vector<Snip> Store::all() const {
  return run_select(db_, "SELECT sid,cid,sidx,txt,q FROM snips ORDER BY cid ASC, sidx ASC;", 0, false);
}

}  // namespace hrm
